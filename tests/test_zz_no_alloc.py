"""The allocation-free 4-step entry point, bfft_hybrid_c2c_noalloc.

Callers that cannot allocate device memory while they run (code inside
another framework's fixed memory pool, loops where cudaMalloc / cudaFree
would synchronise the device, FFI hosts without an allocator for the CUDA
context) use this entry point: it takes only their input and output buffers
and keeps its scratch in a fixed array inside the library.  Its results must
match the regular run_hybrid plan executed through bfft_execute with a
caller workspace, call after call.

This file is collected last on purpose (pytest orders files by name), so a
run that stops at the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from bfft import _lib
from bfft.runner import execute_native, native_plan

from conftest import cplx

pytestmark = pytest.mark.gpu

TOL_REF = 2e-6  # the library's parity tolerance (relative L2)
FWD, INV = 0, 1
NORM = {"none": 0, "forward": 1, "backward": 2, "ortho": 3}


def _noalloc(x, out, n, batch, tile, tdir, norm):
    L = _lib.load()
    st = L.bfft_hybrid_c2c_noalloc(x.data_ptr(), out.data_ptr(), n, batch, tile, tdir, NORM[norm],
                                   x.device.index or 0, torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st, "bfft_hybrid_c2c_noalloc")
    return out


def _regular(x, n, batch, tile, tdir, norm):
    plan = native_plan("run_hybrid", "dit", n, batch, x.device.index or 0, tile=tile, block=256,
                       transform_direction="inverse" if tdir == INV else "forward", norm=norm)
    return execute_native(plan, x, torch.empty_like(x))


def _rel_l2(a, b):
    a = a.cpu().numpy().astype(np.complex128)
    b = b.cpu().numpy().astype(np.complex128)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("cases", [
    [(4096, 64, 64, FWD, "backward"), (65536, 16, 256, INV, "ortho")],
    [(1 << 20, 4, 1024, FWD, "forward"), (2048, 128, 2048, INV, "backward")],
    # one length-N pass (tile 1), a 2-wide first pass (tile < 4: row layout),
    # a 2-point second pass (n / tile < 4: direct stores), and a single-pass
    # shape whose batch * N is past the scratch limit (it uses no scratch)
    [(1024, 8, 1, INV, "ortho"), (4096, 4, 2, FWD, "forward")],
    [(4096, 4, 2048, INV, "backward"), (4096, 2048, 4096, FWD, "none")],
])
def test_noalloc_matches_regular_entry_two_calls_in_a_row(cases):
    rng = np.random.default_rng(77)
    dev = torch.device("cuda:0")
    for n, batch, tile, tdir, norm in cases:
        x = torch.from_numpy(cplx(rng, (batch, n))).to(dev)
        want = _regular(x, n, batch, tile, tdir, norm)
        got = _noalloc(x, torch.empty_like(x), n, batch, tile, tdir, norm)
        torch.cuda.synchronize()
        assert _rel_l2(got, want) <= TOL_REF, (n, batch, tile)
        # the same kernels on the same twiddle values: the same bits
        assert torch.equal(got, want), (n, batch, tile)
        # and it is a transform: check against float64 on one row
        ref = np.fft.fft(x[0].cpu().numpy().astype(np.complex128))
        if tdir == INV:
            ref = np.fft.ifft(x[0].cpu().numpy().astype(np.complex128), norm="forward" if norm == "none" else norm)
        elif norm != "backward":
            ref = np.fft.fft(x[0].cpu().numpy().astype(np.complex128), norm="backward" if norm == "none" else norm)
        row = got[0].cpu().numpy().astype(np.complex128)
        assert np.linalg.norm(row - ref) / np.linalg.norm(ref) <= 1e-6


def test_noalloc_allocates_nothing_and_repeats_bitwise():
    rng = np.random.default_rng(5)
    dev = torch.device("cuda:0")
    n, batch, tile = 16384, 32, 128
    x = torch.from_numpy(cplx(rng, (batch, n))).to(dev)
    a = torch.empty_like(x)
    b = torch.empty_like(x)
    _noalloc(x, a, n, batch, tile, FWD, "backward")  # first call on the device does the set-up
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(dev)[0]
    _noalloc(x, b, n, batch, tile, FWD, "backward")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free_before
    assert torch.equal(a, b)


def test_noalloc_rejects_requests_beyond_its_fixed_scratch():
    dev = torch.device("cuda:0")
    n, batch = 1 << 20, 8  # 2^23 elements > 2^22
    x = torch.zeros((batch, n), dtype=torch.complex64, device=dev)
    before = _lib.launch_counter()
    with pytest.raises(ValueError, match="exceeds the fixed scratch"):
        _noalloc(x, torch.empty_like(x), n, batch, 1024, FWD, "backward")
    assert _lib.launch_counter() == before


def test_no_bounded_wait_expired_in_the_noalloc_passes():
    """The two-pass shapes run the TMA passes, whose mbarrier waits are
    bounded; none of the calls above gave up a wait."""
    assert _lib.device_status(0) == 0
