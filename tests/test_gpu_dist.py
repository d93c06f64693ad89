"""Multi-GPU paths on the device.

* The four phases of ``bfft_dist_phase`` for every rank of P = 1..8, run on
  one GPU with the all-to-alls emulated by device copies, against the host
  restatement (``oracle/dist_oracle.py``) phase by phase, and the assembled
  transform against float64 ``numpy.fft``.
* ``bfft.dist.DistributedFFT`` over NCCL, one process per GPU, when the box
  has 2 or more GPUs.
* Config 5b on one GPU: N = 2^30 as three CTA-resident passes of 2^10,
  checked with float64 DFT bins computed directly, round trip and Parseval.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from bfft import _lib, dist as bdist
from bfft.entry import ExecutionPlan, execute_fft_plan, native_plan_for
from bfft.error_metric import rel_l2_per_transform
from oracle import dist_oracle

from conftest import cplx

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL_F64 = 1e-6


def _native_phase_fns(n1, n2, p, tdir="forward", norm="backward", row_tiles=(0, 0)):
    plans = [_lib.NativeDistPlan(n1, n2, p, r, transform_direction=tdir, norm=norm, row_tiles=row_tiles, device=0)
             for r in range(p)]
    ws = [torch.empty(max(pl.workspace_bytes, 16), dtype=torch.uint8, device=DEV) for pl in plans]
    stream = torch.cuda.current_stream().cuda_stream

    def make(r):
        def fn(k, x):
            x = torch.as_tensor(x, device=DEV).contiguous()
            out = torch.empty_like(x)
            plans[r].phase(k, x.data_ptr(), out.data_ptr(), ws[r].data_ptr(), ws[r].numel(), stream)
            return out
        return fn
    return [make(r) for r in range(p)], plans


def _emulate_device(x, n1, n2, p, tdir="forward", norm="backward", row_tiles=(0, 0), check_phases=True,
                    output_order="natural"):
    """All ranks' native phases with the exchanges done by device slicing;
    each phase is also compared with the host restatement on the same input."""
    fns, _ = _native_phase_fns(n1, n2, p, tdir, norm, row_tiles)
    hosts = [dist_oracle.NumpyPhases(n1, n2, p, r, tdir, norm, dtype=np.complex64) for r in range(p)]
    n = n1 * n2
    slab, chunk = n // p, n // (p * p)
    bufs = [torch.from_numpy(x[r * slab:(r + 1) * slab].copy()).to(DEV) for r in range(p)]
    for k in ((0, 1, 2, 3) if output_order == "natural" else (0, 1, 4)):
        outs = [fns[r](k, bufs[r]) for r in range(p)]
        if check_phases:
            for r in range(p):
                want = hosts[r].phase(k, bufs[r].cpu().numpy())
                got = outs[r].cpu().numpy()
                err = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
                assert err < 1e-6, (n1, n2, p, r, k, err)
        if k in (3, 4):
            return np.concatenate([o.cpu().numpy() for o in outs])
        bufs = [torch.cat([outs[s][r * chunk:(r + 1) * chunk] for s in range(p)]) for r in range(p)]


@pytest.mark.parametrize("n1, n2, p", [(1024, 1024, 1), (1024, 1024, 2), (256, 4096, 4), (4096, 256, 8),
                                       (1 << 15, 1024, 2), (1 << 14, 1 << 13, 4), (64, 64, 8)])
def test_native_phases_emulated_ranks(n1, n2, p):
    rng = np.random.default_rng(n1 + 7 * n2 + p)
    x = cplx(rng, n1 * n2)
    y = _emulate_device(x, n1, n2, p)
    assert rel_l2_per_transform(y, np.fft.fft(x.astype(np.complex128))) <= TOL_F64


@pytest.mark.parametrize("tdir, norm", [("inverse", "backward"), ("forward", "ortho"), ("inverse", "none")])
def test_native_phases_directions_and_norms(tdir, norm):
    rng = np.random.default_rng(3)
    n1, n2, p = 512, 2048, 4
    x = cplx(rng, n1 * n2)
    y = _emulate_device(x, n1, n2, p, tdir, norm, check_phases=False)
    xd = x.astype(np.complex128)
    if tdir == "forward":
        ref = np.fft.fft(xd, norm=norm)
    else:
        ref = np.fft.ifft(xd, norm="forward" if norm == "none" else norm)
    assert rel_l2_per_transform(y, ref) <= TOL_F64


def _ref_transform(x, tdir, norm):
    xd = x.astype(np.complex128)
    if tdir == "forward":
        return np.fft.fft(xd, norm=norm if norm != "none" else "backward")
    return np.fft.ifft(xd, norm=norm if norm != "none" else "forward")


def _transposed_ref(X, n1, n2, p):
    return np.concatenate([dist_oracle.transposed_slab(X, n1, n2, p, r) for r in range(p)])


@pytest.mark.parametrize("n1, n2, p, tdir, norm", [(1024, 1024, 2, "forward", "backward"),
                                                   (256, 4096, 4, "inverse", "backward"),
                                                   (4096, 256, 8, "forward", "ortho"),
                                                   (512, 512, 1, "inverse", "none"),
                                                   (1 << 14, 1 << 13, 4, "forward", "backward")])
def test_native_phases_transposed_output(n1, n2, p, tdir, norm):
    """Transposed-output mode (phase 4 after the second exchange): each phase
    against the host restatement, and every rank's (N1/P) x N2 block against
    the matching columns of float64 numpy.fft."""
    rng = np.random.default_rng(n1 + 5 * n2 + p)
    x = cplx(rng, n1 * n2)
    y = _emulate_device(x, n1, n2, p, tdir, norm, output_order="transposed", check_phases=n1 * n2 <= 1 << 22)
    ref = _transposed_ref(_ref_transform(x, tdir, norm), n1, n2, p)
    assert rel_l2_per_transform(y, ref) <= TOL_F64


def test_distributed_fft_single_rank_and_row_tiles():
    """DistributedFFT without a process group (P = 1), default and explicit
    row-FFT tiles, and the phase launch counts it reports."""
    rng = np.random.default_rng(21)
    n = 1 << 24
    x = cplx(rng, n)
    ref = np.fft.fft(x.astype(np.complex128))
    for tiles in ((0, 0), (64, 4096)):
        f = bdist.DistributedFFT(n, device=DEV, row_tiles=tiles)
        before = _lib.launch_counter()
        y = f.execute(torch.from_numpy(x).to(DEV))
        torch.cuda.synchronize()
        assert _lib.launch_counter() - before == f.launches
        assert rel_l2_per_transform(y.cpu().numpy(), ref) <= TOL_F64, tiles


@pytest.mark.parametrize("output_order", ["natural", "transposed"])
@pytest.mark.parametrize("n1, n2, p, tdir, norm", [(1024, 1024, 2, "forward", "backward"),
                                                   (256, 4096, 4, "inverse", "backward"),
                                                   (4096, 512, 8, "forward", "ortho"), (512, 512, 1, "forward", "none"),
                                                   (1 << 13, 1 << 13, 2, "forward", "backward")])
def test_p2p_phases_emulated_ranks(n1, n2, p, tdir, norm, output_order):
    """Peer-to-peer mode: the exchanges fused into the transposes (stores into
    the other ranks' buffers); all ranks in one process on one GPU, attached
    through device pointers, phases run rank after rank (a barrier between)."""
    rng = np.random.default_rng(n1 * 3 + n2 + p)
    n = n1 * n2
    x = cplx(rng, n)
    plans = [_lib.NativeDistPlan(n1, n2, p, r, transform_direction=tdir, norm=norm, device=0) for r in range(p)]
    bases = [pl.p2p_prepare()[0] for pl in plans]
    for pl in plans:
        pl.p2p_attach_pointers(bases)
    ws = [torch.empty(pl.workspace_bytes, dtype=torch.uint8, device=DEV) for pl in plans]
    st = torch.cuda.current_stream().cuda_stream
    slab = n // p
    xs = [torch.from_numpy(x[r * slab:(r + 1) * slab].copy()).to(DEV) for r in range(p)]
    outs = [torch.empty(slab, dtype=torch.complex64, device=DEV) for _ in range(p)]
    before = _lib.launch_counter()
    for k in ((0, 1, 2, 3) if output_order == "natural" else (0, 1, 4)):
        for r in range(p):
            pl = plans[r]
            pl.p2p_phase(k, xs[r].data_ptr() if k == 0 else 0, outs[r].data_ptr() if k in (3, 4) else 0,
                         ws[r].data_ptr(), ws[r].numel(), st)
    y = torch.cat(outs).cpu().numpy()
    assert _lib.launch_counter() > before
    ref = _ref_transform(x, tdir, norm)
    if output_order == "transposed":
        ref = _transposed_ref(ref, n1, n2, p)
    assert rel_l2_per_transform(y, ref) <= TOL_F64, (n1, n2, p)
    with pytest.raises(ValueError):  # phases before attach are refused
        _lib.NativeDistPlan(n1, n2, p, 0).p2p_phase(1, 0, 0, ws[0].data_ptr(), ws[0].numel(), st)


def test_dist_errors_before_launch():
    with pytest.raises(ValueError):
        _lib.NativeDistPlan(1024, 1024, 3, 0)
    with pytest.raises(ValueError):
        _lib.NativeDistPlan(1024, 1024, 2, 2)
    with pytest.raises(ValueError):
        _lib.NativeDistPlan(1024, 96, 1, 0)
    pl = _lib.NativeDistPlan(64, 64, 1, 0)
    x = torch.zeros(4096, dtype=torch.complex64, device=DEV)
    before = _lib.launch_counter()
    with pytest.raises(ValueError):  # phases 1 and 2 need the workspace
        pl.phase(1, x.data_ptr(), torch.empty_like(x).data_ptr(), 0, 0, 0)
    with pytest.raises(ValueError):
        pl.phase(4, x.data_ptr(), torch.empty_like(x).data_ptr(), 0, 0, 0)
    with pytest.raises(ValueError):  # aliasing
        pl.phase(0, x.data_ptr(), x.data_ptr(), 0, 0, 0)
    assert _lib.launch_counter() == before


# ---------------------------------------------------------------- NCCL, one process per GPU

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


NCCL_CASES = [(1 << 22, "forward", "backward", "p2p", "natural"), (1 << 24, "inverse", "ortho", "p2p", "natural"),
              (1 << 22, "forward", "backward", "nccl", "natural"), (1 << 24, "inverse", "ortho", "nccl", "natural"),
              (1 << 22, "forward", "backward", "p2p", "transposed"),
              (1 << 24, "inverse", "ortho", "nccl", "transposed")]


def _nccl_rank(rank, world, port, results):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        for idx, (n, tdir, norm, mode, order) in enumerate(NCCL_CASES):
            rng = np.random.default_rng(idx % 2)
            x = cplx(rng, n)
            slab = n // world
            f = bdist.DistributedFFT(n, transform_direction=tdir, norm=norm, device=dev, exchange=mode,
                                     output_order=order)
            assert f.exchange == mode
            f.execute(torch.from_numpy(x[rank * slab:(rank + 1) * slab].copy()).to(dev))  # twice: buffer reuse
            y = f.execute(torch.from_numpy(x[rank * slab:(rank + 1) * slab].copy()).to(dev)).cpu().numpy()
            xd = x.astype(np.complex128)
            ref = np.fft.fft(xd, norm=norm) if tdir == "forward" else np.fft.ifft(xd, norm=norm)
            if order == "transposed":
                ref = dist_oracle.transposed_slab(ref, f.n1, f.n2, world, rank)
            else:
                ref = ref[rank * slab:(rank + 1) * slab]
            results[(rank, idx)] = float(np.linalg.norm(y - ref) / np.linalg.norm(ref))
            first, count = bdist.batch_shard(8192)
            results[(rank, "shard")] = (first, count)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_distributed_fft_over_nccl():
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2 or more GPUs in one box")
    world = 4 if ngpu >= 4 else 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_nccl_rank, args=(world, _free_port(), results), nprocs=world, join=True,
                           start_method="spawn")
        res = dict(results)
    for r in range(world):
        for idx in range(len(NCCL_CASES)):
            assert res[(r, idx)] <= TOL_F64, (r, idx, res[(r, idx)])
    shards = sorted(res[(r, "shard")] for r in range(world))
    assert shards[0][0] == 0 and sum(c for _, c in shards) == 8192


# ---------------------------------------------------------------- config 5b on one GPU

def _dft_bins_f64(x: torch.Tensor, bins, chunk=1 << 26):
    """X[k] = sum_n x[n] exp(-2 pi i k n / N) in float64, by direct summation."""
    n = x.numel()
    out = []
    for k in bins:
        acc = torch.zeros((), dtype=torch.complex128, device=x.device)
        for s in range(0, n, chunk):
            idx = torch.arange(s, min(s + chunk, n), device=x.device, dtype=torch.int64)
            ph = ((idx * int(k)) % n).to(torch.float64) * (-2.0 * np.pi / n)
            w = torch.complex(torch.cos(ph), torch.sin(ph))
            acc += (x[s:s + chunk].to(torch.complex128) * w).sum()
            del idx, ph, w
        out.append(acc.item())
    return np.array(out)


@pytest.mark.parametrize("which", ["bench-plan", "tile-1024"])
def test_config5b_single_gpu_n2p30(which):
    """N = 2^30 on one GPU: the plan bench.py times for config 5b (a 128-point
    local group and three tail passes: 7 + 8 + 8 + 7 stages, three-level W_N
    twiddles in the column passes), and a 1024-point local group."""
    n = 1 << 30
    g = torch.Generator(device=DEV).manual_seed(2030)
    x = torch.complex(torch.randn(n, device=DEV, generator=g), torch.randn(n, device=DEV, generator=g))
    if which == "bench-plan":
        import bench

        plan, _ = bench.choose_plan(n, 1)
        assert plan.executed == "fft_dit_matrix" and plan.params["tile"] == 128, plan
        assert native_plan_for(plan, 0).launches == 4
        base = {k: v for k, v in plan.__dict__.items() if k not in ("transform_direction",)}
    else:
        base = dict(n=n, batch=1, direction="dit", precision="fp32", selection_source="table", reason="t",
                    fallback=False, executed="fft_dit_matrix", block=256, params={"tile": 1024})
    fwd = ExecutionPlan(**base)
    y = execute_fft_plan(fwd, x)
    rng = np.random.default_rng(7)
    bins = [0, 1, n // 2, n - 1] + [int(v) for v in rng.integers(0, n, 4)]
    ref = _dft_bins_f64(x, bins)
    got = y[bins].cpu().numpy().astype(np.complex128)
    err = np.sqrt(np.sum(np.abs(got - ref) ** 2) / np.sum(np.abs(ref) ** 2))
    assert err <= TOL_F64, err
    pars = (torch.linalg.vector_norm(y.to(torch.complex128)) ** 2 / n /
            torch.linalg.vector_norm(x.to(torch.complex128)) ** 2).item()
    assert abs(pars - 1) < 1e-5, pars
    inv = ExecutionPlan(**base, transform_direction="inverse")
    back = execute_fft_plan(inv, y)
    del y
    err = (torch.linalg.vector_norm(back - x) / torch.linalg.vector_norm(x)).item()
    assert err <= 2 * TOL_F64, err
    del back, x
    # tone k0 -> N at bin k0
    k0 = 123457
    tone = torch.empty(n, dtype=torch.complex64, device=DEV)
    chunk = 1 << 26
    for s in range(0, n, chunk):
        idx = torch.arange(s, s + chunk, device=DEV, dtype=torch.int64)
        ph = ((idx * k0) % n).to(torch.float64) * (2.0 * np.pi / n)
        tone[s:s + chunk] = torch.complex(torch.cos(ph), torch.sin(ph)).to(torch.complex64)
    yt = execute_fft_plan(fwd, tone)
    peak = yt[k0].item()
    assert abs(peak - n) / n < 1e-6, peak
    yt[k0] = 0
    assert torch.linalg.vector_norm(yt).item() / n < 1e-5
