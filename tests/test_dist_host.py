"""Multi-GPU host logic on CPU ranks (no GPU).

* The batch partition of ``bfft_dist_batch_shard`` (config 5a) covers every
  row exactly once.
* ``bfft.dist.DistributedFFT`` (config 5b) run as ``gloo`` process groups of 2
  and 4 ranks: the real orchestration -- buffer rotation, the three
  ``all_to_all_single`` exchanges and their chunk order -- with the host
  restatement of the device phases (``oracle/dist_oracle.py``) standing in for
  ``bfft_dist_phase``.  Each rank's output slab is compared with float64
  ``numpy.fft`` of the whole input.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from bfft import _build, dist as bdist
from oracle import dist_oracle


@pytest.fixture(scope="module", autouse=True)
def _built():
    _build.build(verbose=False)


@pytest.mark.parametrize("batch", [0, 1, 7, 8, 8192, 8193])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_batch_shard_partitions_rows(batch, world):
    seen = []
    for r in range(world):
        first, count = bdist.batch_shard(batch, world, r)
        assert count in (batch // world, batch // world + 1)
        seen.extend(range(first, first + count))
    assert seen == list(range(batch))


def test_batch_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        bdist.batch_shard(16, 2, 2)
    with pytest.raises(ValueError):
        bdist.batch_shard(-1, 2, 0)


class HostPhases:
    """Host stand-in for the device phases (tests only)."""

    def __init__(self, *args, **kw):
        self.np = dist_oracle.NumpyPhases(*args, **kw, dtype=np.complex64)

    def empty(self, count):
        return torch.empty(count, dtype=torch.complex64)

    def phase(self, k, x, out):
        out.copy_(torch.from_numpy(self.np.phase(k, x.numpy())))


def test_factors_and_validation():
    assert bdist.default_factors(1 << 30) == (1 << 15, 1 << 15)
    assert bdist.default_factors(1 << 11) == (1 << 6, 1 << 5)
    with pytest.raises(ValueError):
        bdist.default_factors(48)
    ph = HostPhases(16, 16, 1, 0)
    f = bdist.DistributedFFT(256, n1=16, phases=ph)
    with pytest.raises(TypeError):
        f.execute(torch.zeros(256, dtype=torch.complex128))
    with pytest.raises(ValueError):
        f.execute(torch.zeros(128, dtype=torch.complex64))
    with pytest.raises(ValueError):
        bdist.DistributedFFT(256, n1=24, phases=ph)
    with pytest.raises(ValueError):
        bdist.DistributedFFT(256, transform_direction="backward", phases=ph)


def test_single_rank_orchestration():
    rng = np.random.default_rng(5)
    n1, n2 = 32, 8
    x = (rng.standard_normal(n1 * n2) + 1j * rng.standard_normal(n1 * n2)).astype(np.complex64)
    f = bdist.DistributedFFT(n1 * n2, n1=n1, phases=HostPhases(n1, n2, 1, 0))
    y = f.execute(torch.from_numpy(x)).numpy()
    ref = np.fft.fft(x.astype(np.complex128))
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        for idx, (n1, n2, tdir, norm, seed, *order) in enumerate(cases):
            order = order[0] if order else "natural"
            n = n1 * n2
            rng = np.random.default_rng(seed)
            x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
            slab = n // world
            f = bdist.DistributedFFT(n, n1=n1, transform_direction=tdir, norm=norm,
                                     phases=HostPhases(n1, n2, world, rank, tdir, norm), output_order=order)
            assert (f.world, f.rank) == (world, rank)
            y = f.execute(torch.from_numpy(x[rank * slab:(rank + 1) * slab].copy()))
            assert f.output_view(y).shape == ((n1 // world, n2) if order == "transposed" else (n2 // world, n1))
            y = y.numpy()
            xd = x.astype(np.complex128)
            ref = np.fft.fft(xd, norm=norm if norm != "none" else "backward") if tdir == "forward" else \
                np.fft.ifft(xd, norm=norm if norm != "none" else "forward")
            if norm == "none" and tdir == "forward":
                ref = np.fft.fft(xd)
            if order == "transposed":
                ref = dist_oracle.transposed_slab(ref, n1, n2, world, rank)
            else:
                ref = ref[rank * slab:(rank + 1) * slab]
            results[(rank, idx)] = float(np.linalg.norm(y - ref) / np.linalg.norm(ref))
    finally:
        dist.destroy_process_group()


CASES = [(32, 32, "forward", "backward", 1), (64, 16, "forward", "ortho", 2), (16, 64, "inverse", "backward", 3),
         (32, 32, "inverse", "forward", 4), (8, 128, "forward", "none", 5),
         # transposed-output mode: two exchanges, each rank ends with whole columns k1
         (32, 32, "forward", "backward", 6, "transposed"), (16, 64, "inverse", "ortho", 7, "transposed"),
         (64, 16, "inverse", "none", 8, "transposed")]


@pytest.mark.parametrize("world", [2, 4])
def test_distributed_4step_over_gloo(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), CASES, results), nprocs=world,
                           join=True, start_method="spawn")
        res = dict(results)
    assert len(res) == world * len(CASES)
    for key, err in res.items():
        assert err < 1e-6, (key, err)


def test_emulated_ranks_match_numpy():
    """The same phases with the exchanges done by slicing (the emulation the
    single-GPU device test uses) give the transform for P = 1..8."""
    rng = np.random.default_rng(11)
    for n1, n2, p in [(16, 16, 1), (16, 16, 2), (64, 32, 4), (128, 8, 8)]:
        n = n1 * n2
        x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
        y = dist_oracle.emulate(x, n1, n2, p)
        assert np.linalg.norm(y - np.fft.fft(x)) / np.linalg.norm(y) < 1e-12
        yt = dist_oracle.emulate(x, n1, n2, p, output_order="transposed")
        ref = np.concatenate([dist_oracle.transposed_slab(np.fft.fft(x), n1, n2, p, r) for r in range(p)])
        assert np.linalg.norm(yt - ref) / np.linalg.norm(ref) < 1e-12


def test_output_order_validation():
    ph = HostPhases(16, 16, 1, 0)
    with pytest.raises(ValueError):
        bdist.DistributedFFT(256, n1=16, phases=ph, output_order="bitreversed")
    f = bdist.DistributedFFT(256, n1=16, phases=ph, output_order="transposed")
    x = (np.arange(256) * (1 + 0.5j)).astype(np.complex64)
    y = f.execute(torch.from_numpy(x)).numpy()
    ref = np.fft.fft(x.astype(np.complex128)).reshape(16, 16).T.reshape(-1)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6
