"""The tensor-core 16-point row DFT (bfft_tc_dft16_rows, 3xTF32 tcgen05.mma).

The reference's dense-dot core (src/xpu/kernels.py:487-532) multiplies tiles
of rows by the tile's DFT matrix with FP32 dots; this kernel does the same
product on the tensor cores with the 3xTF32 split.  Its results must stay
within 1e-6 relative L2 of float64 numpy (the library's float64 bound) and
next to the FP32 row path, for full tiles, ragged tails and single rows, both
directions.
"""
import numpy as np
import pytest
import torch

from bfft import _lib
from bfft.tc_experiment import rel_l2_f64, tc_rows

from conftest import cplx

pytestmark = pytest.mark.gpu

TOL_F64 = 1e-6  # relative L2 against float64


@pytest.mark.parametrize("rows", [1, 127, 128, 129, 1000, 4096 + 77])
@pytest.mark.parametrize("inverse", [False, True])
def test_tc_dft16_rows_vs_float64(rows, inverse):
    rng = np.random.default_rng(1600 + rows + (7 if inverse else 0))
    xh = cplx(rng, (rows, 16))
    x = torch.from_numpy(xh).cuda()
    # the output starts as NaN so rows the kernel misses show up
    y = torch.full_like(x, complex(float("nan"), float("nan")))
    _lib.device_status(0, clear=True)
    tc_rows(x, y, inverse, 1.0 / 16 if inverse else 1.0)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.isfinite(got.view(np.float32)).all()
    err = rel_l2_f64(got, xh, inverse)
    assert err <= TOL_F64, err
    assert _lib.device_status(0) == 0


def test_tc_dft16_rows_large_batch_and_scale():
    rows = 1 << 18
    rng = np.random.default_rng(1616)
    xh = cplx(rng, (rows, 16)) * np.float32(1e3)
    x = torch.from_numpy(xh).cuda()
    y = torch.empty_like(x)
    tc_rows(x, y, False, 0.25)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = np.fft.fft(xh.astype(np.complex128), axis=-1) * 0.25
    err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err <= TOL_F64, err
    # the same bytes on a second call (no state carried between tiles)
    y2 = torch.empty_like(x)
    tc_rows(x, y2, False, 0.25)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


def test_tc_dft16_rows_rejects_bad_arguments():
    L = _lib.load()
    x = torch.zeros(64, 16, dtype=torch.complex64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert L.bfft_tc_dft16_rows(x.data_ptr(), x.data_ptr(), 64, 0, 1.0, 0, s) != 0  # aliasing
    y = torch.zeros_like(x)
    assert L.bfft_tc_dft16_rows(x.data_ptr(), y.data_ptr(), 0, 0, 1.0, 0, s) != 0  # no rows
    assert L.bfft_tc_dft16_rows(x.data_ptr() + 8, y.data_ptr(), 63, 0, 1.0, 0, s) != 0  # 8-byte aligned only
    assert L.bfft_tc_dft16_rows(x.data_ptr(), y.data_ptr(), 64, 5, 1.0, 0, s) != 0  # bad direction
