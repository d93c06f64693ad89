"""GPU parity of libbfft (B200) against the reference and float64.

Tolerances: relative L2 <= 2e-6 against the
reference's own implementation of each path (golden vectors produced by the
reference), <= 1e-6 per transform against float64 numpy; index maps and
permutations bit-exact.  Every call goes through the public API and the C ABI.
"""
import numpy as np
import pytest
import torch

import bfft
from bfft import _lib, runner
from bfft.adapter_hybrid import plan_hybrid, run_hybrid
from bfft.entry import ExecutionPlan, execute_fft_plan
from bfft.error_metric import rel_l2, rel_l2_per_transform
from oracle import oracle as O

from conftest import cplx

pytestmark = pytest.mark.gpu

TOL_REF = 2e-6
TOL_F64 = 1e-6
DEV = "cuda:0"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---------------------------------------------------------------- index maps

@pytest.mark.parametrize("kind", [0, 1, 2])
def test_device_index_maps_bit_exact(kind):
    L = _lib.load()
    name = ("bitrev", "dit_digrev", "dif_digrev")[kind]
    for bits in list(range(0, 13)) + [16, 20]:
        out = torch.empty(1 << bits, dtype=torch.int32, device=DEV)
        _lib.check(L.bfft_index_map(kind, bits, out.data_ptr(), 0, torch.cuda.current_stream().cuda_stream))
        got = host(out).view(np.uint32)
        want = O.index_table(name, bits) if bits else np.zeros(1, np.uint32)
        np.testing.assert_array_equal(got, want, err_msg=f"{name} bits={bits}")


def test_device_index_maps_match_reference_kernels(golden):
    L = _lib.load()
    for kind, name in enumerate(("bitrev", "dit_digrev", "dif_digrev")):
        for bits in range(1, 13):
            out = torch.empty(1 << bits, dtype=torch.int32, device=DEV)
            _lib.check(L.bfft_index_map(kind, bits, out.data_ptr(), 0, 0))
            np.testing.assert_array_equal(host(out).view(np.uint32), golden[f"idx_{name}_{bits}"])


def test_bit_reverse_permute_bit_exact(golden):
    for n in (8, 64, 1024):
        x = np.arange(n, dtype=np.float32).astype(np.complex64)
        np.testing.assert_array_equal(host(runner.bit_reverse_permute(dev(x))), golden[f"bitrev_permute_{n}"])
    rng = np.random.default_rng(1)
    x = cplx(rng, (4, 1 << 14))
    got = host(runner.bit_reverse_permute(dev(x)))
    np.testing.assert_array_equal(got.view(np.uint64), O.bitrev_permute(x).view(np.uint64))


# ---------------------------------------------------------------- golden replay

_KNOBS = ("tile", "rows", "glog", "maxp", "cells", "variant")


def _run_case(c, x):
    r = c.get("runner")
    t = dev(x)
    if "plan" in c:
        p = c["plan"]
        plan = ExecutionPlan(n=c["n"], batch=c["batch"], direction="dit", precision="fp32",
                             selection_source="table", reason="golden replay", fallback=p["fallback"],
                             executed=p["executed"], block=256, params=p["params"],
                             transform_type=p["transform_type"],
                             transform_direction=p["transform_direction"], norm=p["norm"])
        return execute_fft_plan(plan, t)
    if r == "r2c_stitch":
        return runner.r2c_stitch(t, c["n"], scale=c["scale"])
    if r == "c2r_pre":
        return runner.c2r_pre(t, c["n"])
    if r == "c2r_unpack":
        return runner.c2r_unpack(t, c["n"], scale=c["scale"])
    if r == "run_hybrid":
        return run_hybrid(t, plan_hybrid(c["n"], c["batch"], tile=c["tile"]))
    fn = getattr(runner, r)
    kw = {k: c[k] for k in _KNOBS if k in c}
    return fn(t, block=256, **kw)


def test_golden_replay_every_reference_case(golden, golden_meta):
    seen = 0
    for c in golden_meta["cases"]:
        lab = c["label"]
        x, want = golden[lab + "__in"], golden[lab + "__out"]
        got = host(_run_case(c, x))
        assert got.shape == want.shape and got.dtype == want.dtype, (lab, got.shape, want.shape)
        e = rel_l2(got, want)
        assert e <= TOL_REF, (lab, e)
        seen += 1
    assert seen >= 50


# ---------------------------------------------------------------- sweeps vs float64

RANK1 = ["fft_dit", "fft_dif", "fft_dit_radix4", "fft_dif_radix4", "fft_dit_fused", "fft_dit_matrix",
         "fft_dif_matrix", "fft_dit_grouped", "fft_dif_grouped"]
BATCHED = ["fft_dit_batch", "fft_dif_batch", "fft_dit_radix4_batch", "fft_dif_radix4_batch",
           "fft_dit_matrix_batch", "fft_dif_matrix_batch"]


def _f64(x):
    return np.fft.fft(x.astype(np.complex128), axis=-1)


@pytest.mark.parametrize("name", RANK1)
def test_rank1_runner_sweep(name):
    rng = np.random.default_rng(hash(name) & 0xFFFF)
    for log2n in range(1, 17):
        n = 1 << log2n
        if "radix4" in name and n < 4:
            continue
        x = cplx(rng, n)
        kw = {}
        if name in ("fft_dit_fused", "fft_dit_matrix", "fft_dif_matrix", "fft_dit_grouped", "fft_dif_grouped"):
            kw["tile"] = 64 if name != "fft_dit_grouped" and name != "fft_dif_grouped" else 8
        got = host(getattr(runner, name)(dev(x), block=256, **kw))
        assert rel_l2(got, _f64(x)) <= TOL_F64, (name, n)


@pytest.mark.parametrize("name", BATCHED)
def test_batched_runner_sweep(name):
    rng = np.random.default_rng(len(name))
    variants = ["spread", "folded"] if name in ("fft_dit_batch", "fft_dif_batch") else ["spread"]
    for log2n in range(1, 15):
        n = 1 << log2n
        if "radix4" in name and n < 4:
            continue
        for b in (1, 4, 32):
            x = cplx(rng, (b, n))
            for v in variants:
                kw = {"variant": v}
                if "matrix" in name:
                    kw["tile"] = min(n, 4096) if log2n % 2 else 64
                got = host(getattr(runner, name)(dev(x), block=128, **kw))
                assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (name, n, b, v)


@pytest.mark.parametrize("tile", [2, 16, 64, 4096])
def test_local_fused_core_two_pass_sizes(tile):
    rng = np.random.default_rng(tile)
    for log2n in (13, 16, 18, 20):
        n = 1 << log2n
        b = max(1, (1 << 21) // n)
        x = cplx(rng, (b, n))
        for name in ("fft_dit_matrix_batch", "fft_dif_matrix_batch"):
            got = host(getattr(runner, name)(dev(x), tile=tile))
            assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (name, n, tile)


@pytest.mark.parametrize("tile", [2, 8, 64, 1024, 4096])
def test_run_hybrid_factorisations(tile):
    rng = np.random.default_rng(tile + 1)
    for n in (4096, 1 << 16, 1 << 20):
        if n // tile > 4096 or tile > n:
            continue
        b = max(1, (1 << 21) // n)
        x = cplx(rng, (b, n))
        got = host(run_hybrid(dev(x), plan_hybrid(n, b, tile=tile)))
        assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (n, tile)


# ---------------------------------------------------------------- semantics

def _plan(executed, n, b, **kw):
    base = dict(n=n, batch=b, direction="dit", precision="fp32", selection_source="table", reason="t",
                fallback=False, executed=executed, block=256)
    base.update(kw)
    return ExecutionPlan(**base)


@pytest.mark.parametrize("executed, params", [("fft_dit_batch", {"variant": "folded"}),
                                               ("fft_dit_matrix_batch", {"tile": 1024}),
                                               ("fft_dif_radix4_batch", {})])
@pytest.mark.parametrize("norm", ["none", "forward", "backward", "ortho"])
def test_c2c_norms_and_directions(executed, params, norm):
    rng = np.random.default_rng(2)
    n, b = 1024, 16
    x = cplx(rng, (b, n))
    t = dev(x)
    xt = torch.from_numpy(x)
    for tdir in ("forward", "inverse"):
        y = host(execute_fft_plan(_plan(executed, n, b, params=params, transform_direction=tdir, norm=norm), t))
        if tdir == "forward":
            ref = torch.fft.fft(xt.to(torch.complex128), norm=None if norm == "none" else norm)
            if norm == "none":
                ref = torch.fft.fft(xt.to(torch.complex128))
        else:
            ref = torch.fft.ifft(xt.to(torch.complex128), norm="forward" if norm == "none" else norm)
        assert rel_l2_per_transform(y, ref.numpy()) <= TOL_F64, (tdir, norm)


@pytest.mark.parametrize("n, b", [(4, 1), (64, 1), (256, 16), (4096, 16), (16384, 4), (1 << 17, 2)])
@pytest.mark.parametrize("norm", ["backward", "forward", "ortho", "none"])
@pytest.mark.parametrize("dedicated", [True, False])
def test_real_flows(n, b, norm, dedicated):
    rng = np.random.default_rng(n + b)
    shape = (n,) if b == 1 else (b, n)
    x = rng.standard_normal(shape).astype(np.float32)
    params = {"real_flow": "dedicated-r2c-pack-v1"} if dedicated else {"real_compat": "packed-c2c-compat"}
    runner_name = "fft_dit_matrix_batch" if b > 1 else "fft_dit_matrix"
    params["tile"] = min(max(n // (2 if dedicated else 1), 1), 4096)
    p = _plan(runner_name, n, b, transform_type="r2c", norm=norm, params=params)
    y = host(execute_fft_plan(p, dev(x)))
    ref = np.fft.rfft(x.astype(np.float64), norm=None if norm == "none" else norm)
    assert rel_l2_per_transform(y, ref) <= TOL_F64, ("r2c", n, b, norm, dedicated)
    xh = np.fft.rfft(rng.standard_normal(shape)).astype(np.complex64)
    xh[..., 0] += 3j   # DC / Nyquist imaginary parts are ignored (torch.fft contract)
    xh[..., -1] -= 2j
    cparams = dict(params)
    if dedicated:
        cparams["real_flow"] = "dedicated-c2r-hermitian-v1"
    pc = _plan(runner_name, n, b, transform_type="c2r", transform_direction="inverse", norm=norm, params=cparams)
    r = host(execute_fft_plan(pc, dev(xh)))
    clean = xh.astype(np.complex128).copy()
    clean[..., 0] = clean[..., 0].real
    clean[..., -1] = clean[..., -1].real
    ref = np.fft.irfft(clean, n=n, norm="forward" if norm == "none" else norm)
    assert r.dtype == np.float32 and r.shape == shape
    assert rel_l2_per_transform(r, ref) <= TOL_F64, ("c2r", n, b, norm, dedicated)


@pytest.mark.parametrize("n", [4096, 16384, 65536])
@pytest.mark.parametrize("flow", ["product", "dedicated", "compat"])
def test_config4_full_shape(n, flow):
    """Config 4 at its exact shape (B = 256): the plan bench.py times
    ("product": the selector's choice, or the explicit dedicated flow when it
    abstains), the dedicated flow with a 256-point local group, and the packed
    C2C compat flow; every row against float64."""
    import bench

    b = 256
    rng = np.random.default_rng(n)
    x = rng.standard_normal((b, n)).astype(np.float32)
    xh = np.fft.rfft(rng.standard_normal((b, n)).astype(np.float32).astype(np.float64)).astype(np.complex64)
    for tt, td, inp in (("r2c", "forward", x), ("c2r", "inverse", xh)):
        if flow == "product":
            p, _ = bench.choose_plan(n, b, tt, td)
        else:
            rf = "dedicated-r2c-pack-v1" if tt == "r2c" else "dedicated-c2r-hermitian-v1"
            params = {"real_flow": rf} if flow == "dedicated" else {"real_compat": "packed-c2c-compat"}
            params.update(tile=256, batch=b, variant="spread")
            p = _plan("fft_dit_matrix_batch", n, b, transform_type=tt, transform_direction=td, params=params)
        got = host(execute_fft_plan(p, dev(inp)))
        if tt == "r2c":
            ref = np.fft.rfft(inp.astype(np.float64), axis=-1)
        else:
            ref = np.fft.irfft(inp.astype(np.complex128), n=n, axis=-1)
        assert got.shape == ref.shape, (tt, got.shape)
        assert rel_l2_per_transform(got, ref) <= TOL_F64, (tt, flow, p.executed, p.params)


@pytest.mark.parametrize("n", [1024, 2048])
def test_config2_full_shape(n):
    """Config 2 at B = 64: forward, inverse (1/N) and the round trip through
    the plans bench.py times, every row against float64."""
    import bench

    b = 64
    rng = np.random.default_rng(n + 64)
    x = cplx(rng, (b, n))
    pf, _ = bench.choose_plan(n, b, "c2c", "forward")
    pi, _ = bench.choose_plan(n, b, "c2c", "inverse")
    t = dev(x)
    y = execute_fft_plan(pf, t)
    back = execute_fft_plan(pi, y)
    x64 = x.astype(np.complex128)
    assert rel_l2_per_transform(host(y), np.fft.fft(x64, axis=-1)) <= TOL_F64
    assert rel_l2_per_transform(host(execute_fft_plan(pi, t)), np.fft.ifft(x64, axis=-1)) <= TOL_F64
    assert rel_l2_per_transform(host(back), x64) <= 2 * TOL_F64


def test_run_fft_public_api_and_squeeze():
    rng = np.random.default_rng(4)
    x = cplx(rng, (1, 2048))
    y, rep = bfft.run_fft(dev(x), "dit", profile_hash=None)
    assert tuple(y.shape) == (1, 2048) and rep.fallback and rep.executed == "fft_dit"
    assert rel_l2(host(y), _f64(x)) <= TOL_F64
    xb = cplx(rng, (16, 1024))
    y2, rep2 = bfft.run_fft(dev(xb), "dif", transform_direction="inverse")
    assert rep2.executed == "fft_dif_batch"
    assert rel_l2_per_transform(host(y2), np.fft.ifft(xb.astype(np.complex128))) <= TOL_F64
    xr = rng.standard_normal(4096).astype(np.float32)
    yr, _ = bfft.run_fft(dev(xr), "dit", transform_type="r2c")
    assert rel_l2(host(yr), np.fft.rfft(xr.astype(np.float64))) <= TOL_F64
    back, rep3 = bfft.run_fft(yr, "dit", transform_type="c2r")
    assert rep3.n == 4096 and rel_l2(host(back), xr) <= TOL_F64


def test_plan_reuse_is_bitwise_stable():
    rng = np.random.default_rng(6)
    x = dev(cplx(rng, (64, 2048)))
    p = _plan("fft_dit_matrix_batch", 2048, 64, params={"tile": 2048})
    a = host(execute_fft_plan(p, x))
    for _ in range(3):
        np.testing.assert_array_equal(host(execute_fft_plan(p, x)).view(np.uint64), a.view(np.uint64))


def test_edge_sizes():
    rng = np.random.default_rng(8)
    for n in (1, 2, 4):
        x = cplx(rng, n)
        y = host(execute_fft_plan(_plan("fft_dit", n, 1), dev(x)))
        assert rel_l2(y, _f64(x)) <= TOL_F64
        yi = host(execute_fft_plan(_plan("fft_dit", n, 1, transform_direction="inverse"), dev(x)))
        assert rel_l2(yi, np.fft.ifft(x.astype(np.complex128))) <= TOL_F64
    # batch=1 batched runner == rank-1 runner
    x = cplx(rng, 4096)
    a = host(runner.fft_dit_matrix(dev(x), tile=4096))
    b = host(runner.fft_dit_matrix_batch(dev(x[None]), tile=4096))[0]
    np.testing.assert_array_equal(a.view(np.uint64), b.view(np.uint64))


def test_errors_raise_before_any_launch():
    before = _lib.launch_counter()
    p = _plan("fft_dit", 1024, 1)
    with pytest.raises(TypeError):
        execute_fft_plan(p, torch.zeros(1024, dtype=torch.complex128, device=DEV))
    with pytest.raises(ValueError):
        execute_fft_plan(p, torch.zeros(512, dtype=torch.complex64, device=DEV))
    with pytest.raises(ValueError):
        execute_fft_plan(p, torch.zeros(1024, dtype=torch.complex64))  # host tensor
    with pytest.raises(ValueError):
        execute_fft_plan(p, torch.zeros(2048, dtype=torch.complex64, device=DEV)[::2])
    with pytest.raises(ValueError):
        runner.fft_dit(torch.zeros(1000, dtype=torch.complex64, device=DEV))
    with pytest.raises(ValueError):
        runner.fft_dit_batch(torch.zeros(3, 8, dtype=torch.complex64, device=DEV))
    with pytest.raises(ValueError):
        runner.fft_dit_matrix_batch(torch.zeros(4, 8, dtype=torch.complex64, device=DEV), variant="folded")
    torch.cuda.synchronize()
    assert _lib.launch_counter() == before


# ---------------------------------------------------------------- full-size properties

def test_sweep_config_full_size_properties():
    """Config 3 at full size (B*N = 2^24): round trip, Parseval and linearity on
    the device, plus sampled transforms against float64."""
    g = torch.Generator(device=DEV).manual_seed(1234)
    for log2n in (4, 8, 12, 16, 20):
        n = 1 << log2n
        b = (1 << 24) // n
        x = torch.complex(torch.randn(b, n, device=DEV, generator=g), torch.randn(b, n, device=DEV, generator=g))
        tile = min(n, 4096)
        fwd = _plan("fft_dit_matrix_batch", n, b, params={"tile": tile})
        inv = _plan("fft_dit_matrix_batch", n, b, params={"tile": tile}, transform_direction="inverse")
        y = execute_fft_plan(fwd, x)
        back = execute_fft_plan(inv, y)
        err = (torch.linalg.vector_norm(back - x) / torch.linalg.vector_norm(x)).item()
        assert err <= 2 * TOL_F64, (n, err)
        pars = (torch.linalg.vector_norm(y.to(torch.complex128)) ** 2 / n / torch.linalg.vector_norm(x.to(torch.complex128)) ** 2).item()
        assert abs(pars - 1) < 1e-5, (n, pars)
        y2 = execute_fft_plan(fwd, 2 * x + 0.5j * x)
        lin = (torch.linalg.vector_norm(y2 - (2 + 0.5j) * y) / torch.linalg.vector_norm(y2)).item()
        assert lin < 1e-6, (n, lin)
        rows = [0, b // 2, b - 1]
        xs = x[rows].cpu().numpy()
        assert rel_l2_per_transform(y[rows].cpu().numpy(), _f64(xs)) <= TOL_F64, n
        del x, y, back, y2


@pytest.mark.parametrize("tile", [256, 65536])
def test_batch_shard_config_full_size(tile):
    """Config 5a on one GPU: N=65536, B=8192 (4 GiB), as two passes (tile 256)
    and as the fused single pass (tile = N): round trip on device and sampled
    rows against float64."""
    n, b = 65536, 8192
    g = torch.Generator(device=DEV).manual_seed(99)
    x = torch.complex(torch.randn(b, n, device=DEV, generator=g), torch.randn(b, n, device=DEV, generator=g))
    fwd = _plan("fft_dit_matrix_batch", n, b, params={"tile": tile})
    y = execute_fft_plan(fwd, x)
    rows = [0, 1, 4095, 8191]
    assert rel_l2_per_transform(y[rows].cpu().numpy(), _f64(x[rows].cpu().numpy())) <= TOL_F64
    back = execute_fft_plan(_plan("fft_dit_matrix_batch", n, b, params={"tile": tile},
                                  transform_direction="inverse"), y)
    err = (torch.linalg.vector_norm(back - x) / torch.linalg.vector_norm(x)).item()
    assert err <= 2 * TOL_F64
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("log2n", [13, 14, 15, 16, 17, 18, 19, 20])
def test_fused_single_pass_batches_and_ring_reuse(log2n):
    """The fused single pass (tile = N, batch >= 2): ragged batches, and a batch
    past the scratch ring so slots are reused (the ring holds 48 MiB: 96
    transforms at 2^16 .. 768 at 2^13, 6 at 2^20 with the 256-consumer tiles);
    forward against float64 on every row, inverse with ortho norm against
    float64, one launch per call, and no bounded wait expired."""
    from bfft.entry import native_plan_for

    n = 1 << log2n
    ring = 3072 * 16384 // (8 * n)
    rng = np.random.default_rng(100 + log2n)
    for b in ((2, 3, 37, ring + 45) if log2n <= 16 else (2, 3, ring + 5)):
        x = cplx(rng, (b, n))
        t = dev(x)
        p = _plan("fft_dit_matrix_batch", n, b, params={"tile": n})
        assert native_plan_for(p, 0).launches == 1
        got = host(execute_fft_plan(p, t))
        assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (n, b)
        pi = _plan("fft_dit_matrix_batch", n, b, params={"tile": n}, transform_direction="inverse", norm="ortho")
        yi = host(execute_fft_plan(pi, t))
        assert rel_l2_per_transform(yi, np.fft.ifft(x.astype(np.complex128), norm="ortho")) <= TOL_F64, (n, b)
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("log2n", [13, 14, 15, 16])
def test_cluster_single_pass(log2n):
    """Whole transforms of 2^13..2^16 points in one HBM round trip (thread-block
    cluster, transpose through distributed shared memory): M2 with tile = N."""
    n = 1 << log2n
    rng = np.random.default_rng(log2n)
    for b in (1, 2, 64):
        x = cplx(rng, (b, n))
        t = dev(x)
        for direction in ("dit", "dif"):
            name = f"fft_{direction}_matrix_batch"
            got = host(getattr(runner, name)(t, tile=n))
            assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (n, b, direction)
        p = _plan("fft_dit_matrix_batch", n, b, params={"tile": n}, transform_direction="inverse", norm="ortho")
        y = host(execute_fft_plan(p, t if b > 1 else t[0])).reshape(b, n)
        ref = np.fft.ifft(x.astype(np.complex128), norm="ortho")
        assert rel_l2_per_transform(y, ref) <= TOL_F64, (n, b, "inverse")
    from bfft.entry import native_plan_for

    assert native_plan_for(_plan("fft_dit_matrix_batch", n, 64, params={"tile": n}), 0).launches == 1


def test_installed_b200_table_selects_and_executes():
    """The committed B200 selector table binds this environment: plan_fft with
    the live profile selects measured entries (legacy and semantic tiers) and
    they execute within tolerance."""
    from bfft.config import DeviceProfile
    from bfft.envcheck import current_env_hash
    from bfft.selector import load_table

    table = load_table()
    if current_env_hash() != table["env_hash"]:
        pytest.skip(f"selector table bound to env {table['env_hash']}, this box is {current_env_hash()}: "
                    "re-measure with python -m bfft.table_builder")
    ph = DeviceProfile.load().hash()
    rng = np.random.default_rng(8)
    for n, b, tt, td in [(2048, 1, "c2c", "forward"), (1024, 16, "c2c", "inverse"), (65536, 8192 // 64, "c2c", "forward"),
                         (4096, 256, "r2c", "forward"), (16384, 256, "c2r", "inverse")]:
        p = bfft.plan_fft("dit", n, batch=b, profile_hash=ph, transform_type=tt, transform_direction=td)
        if (n, b) != (65536, 128):
            assert not p.fallback and p.selection_source == "table", (n, b, tt, p.reason)
        if tt == "r2c":
            x = rng.standard_normal((b, n)).astype(np.float32)
            ref = np.fft.rfft(x.astype(np.float64))
        elif tt == "c2r":
            x = np.fft.rfft(rng.standard_normal((b, n))).astype(np.complex64)
            ref = np.fft.irfft(x.astype(np.complex128), n=n)
        else:
            x = cplx(rng, (b, n))
            ref = np.fft.fft(x.astype(np.complex128)) if td == "forward" else np.fft.ifft(x.astype(np.complex128))
        t = dev(x if b > 1 else x[0])
        y = host(execute_fft_plan(p, t)).reshape(ref.shape)
        assert rel_l2_per_transform(y, ref) <= TOL_F64, (n, b, tt, p.executed)


@pytest.mark.parametrize("n, tiles", [(16, (16,)), (32, (32,)), (64, (64,)), (128, (128,)), (256, (256,)),
                                      (512, (512,)), (1024, (1024,)), (2048, (2048,)), (4096, (4096,)),
                                      (8192, (256, 512)),
                                      (65536, (256,)), (1 << 18, (64, 512))])
def test_tma_passes_odd_batches(n, tiles):
    """The row-pair kernel and the bulk-copy row pass (partial last tiles when
    B is not a multiple of the rows per tile; padded per-row copies below 256
    points and in the row-pair stages of 256 and 1024 points) and the TMA
    column pass (every tail pass, strided local groups), both directions,
    forward and ortho inverse."""
    rng = np.random.default_rng(n)
    for b in (1, 2, 8):  # the runner functions take power-of-two batches (the reference's rule)
        x = cplx(rng, (b, n))
        t = dev(x)
        for tile in tiles:
            for name in ("fft_dit_matrix_batch", "fft_dif_matrix_batch"):
                got = host(getattr(runner, name)(t, tile=tile)).reshape(b, n)
                assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (name, n, b, tile)
    for b in (1, 3, 17):  # plans take any batch
        x = cplx(rng, (b, n))
        t = dev(x)
        for tile in tiles:
            fwd = _plan("fft_dif_matrix_batch", n, b, params={"tile": tile})
            got = host(execute_fft_plan(fwd, t if b > 1 else t[0])).reshape(b, n)
            assert rel_l2_per_transform(got, _f64(x)) <= TOL_F64, (n, b, tile, "dif")
            p = _plan("fft_dit_matrix_batch", n, b, params={"tile": tile}, transform_direction="inverse",
                      norm="ortho")
            y = host(execute_fft_plan(p, t if b > 1 else t[0])).reshape(b, n)
            ref = np.fft.ifft(x.astype(np.complex128), norm="ortho")
            assert rel_l2_per_transform(y, ref) <= TOL_F64, (n, b, tile, "inverse")
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("n, b, tile", [(64, 64, 64), (1024, 8, 1024), (65536, 4, 256), (1 << 18, 2, 512)])
def test_unaligned_buffers_take_the_fallback_pass(n, b, tile):
    """Input, output and workspace 8 but not 16 bytes aligned: the TMA column
    pass and the bulk-copy row pass need 16-byte aligned buffers, so the
    library runs these passes on its cp.async pass instead -- the results are
    as accurate as from aligned buffers."""
    rng = np.random.default_rng(n + b)
    x = cplx(rng, (b, n))
    plan = runner.native_plan("fft_dit_matrix_batch", "dit", n, b, 0, tile=tile, block=256)
    xin = torch.empty(b * n + 1, dtype=torch.complex64, device=DEV)
    xin[1:].copy_(torch.from_numpy(x).reshape(-1))
    out = torch.zeros(b * n + 1, dtype=torch.complex64, device=DEV)
    ws = torch.empty(plan.workspace_bytes + 8, dtype=torch.uint8, device=DEV) if plan.workspace_bytes else None
    assert xin[1:].data_ptr() % 16 == 8 and out[1:].data_ptr() % 16 == 8
    plan.execute(xin[1:].data_ptr(), out[1:].data_ptr(), ws.data_ptr() + 8 if ws is not None else 0,
                 plan.workspace_bytes, torch.cuda.current_stream(DEV).cuda_stream)
    y = host(out[1:]).reshape(b, n)
    assert rel_l2_per_transform(y, _f64(x)) <= TOL_F64, (n, b, tile)
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("n, b, tt, chunks", [(1024, 64, "c2c", 4), (65536, 32, "c2c", 8), (4096, 16, "r2c", 4),
                                             (4096, 16, "c2r", 2), (2048, 1, "c2c", 1)])
def test_host_buffer_execution(n, b, tt, chunks):
    """execute_fft_plan_host (chunked, copies overlapped with the transform on
    three streams) equals the device path bit for bit and float64 within
    tolerance."""
    from bfft.host_io import execute_fft_plan_host

    rng = np.random.default_rng(n + b)
    if tt == "r2c":
        x = rng.standard_normal((b, n)).astype(np.float32)
        ref = np.fft.rfft(x.astype(np.float64))
        p = _plan("fft_dif_matrix_batch", n, b, params={"tile": n // 2, "real_flow": "dedicated-r2c-pack-v1"},
                  transform_type="r2c")
    elif tt == "c2r":
        x = np.fft.rfft(rng.standard_normal((b, n))).astype(np.complex64)
        ref = np.fft.irfft(x.astype(np.complex128), n=n)
        p = _plan("fft_dit_matrix_batch", n, b, params={"tile": n // 2, "real_flow": "dedicated-c2r-hermitian-v1"},
                  transform_type="c2r", transform_direction="inverse")
    else:
        x = cplx(rng, (b, n))
        ref = np.fft.fft(x.astype(np.complex128))
        p = _plan("fft_dit_matrix_batch" if b > 1 else "fft_dit_matrix", n, b, params={"tile": min(n, 256)})
    xt = torch.from_numpy(x if b > 1 else x[0]).pin_memory()
    got = execute_fft_plan_host(p, xt, chunks=chunks).numpy()
    dev_out = host(execute_fft_plan(p, xt.cuda()))
    assert np.array_equal(got, dev_out)
    assert rel_l2_per_transform(got.reshape(ref.shape), ref) <= TOL_F64


def test_installed_composition_table_selects_and_executes():
    """The promoted exact-shape 4-step entries resolve through plan_fft as
    selection_source='composition' (run_hybrid) and execute within tolerance;
    shapes without an entry keep the selector's plan."""
    from bfft.composition import load_composition_table
    from bfft.config import DeviceProfile
    from bfft.envcheck import current_env_hash

    comp = load_composition_table()
    if comp is None:
        pytest.skip("no composition promoted on this stack")
    if current_env_hash() != comp["env_hash"]:
        pytest.skip(f"composition table bound to env {comp['env_hash']}, this box is {current_env_hash()}")
    ph = DeviceProfile.load().hash()
    rng = np.random.default_rng(12)
    for e in comp["entries"]:
        n, b = e["N"], e["batch"]
        p = bfft.plan_fft("dit", n, batch=b, profile_hash=ph)
        assert p.selection_source == "composition" and p.executed == "run_hybrid" and p.params["tile"] == e["tile"]
        x = cplx(rng, (b, n))
        y = host(execute_fft_plan(p, dev(x if b > 1 else x[0]))).reshape(b, n)
        assert rel_l2_per_transform(y, _f64(x)) <= TOL_F64, (n, b)
    p = bfft.plan_fft("dit", 2048, batch=16, profile_hash=ph)
    assert p.selection_source == "table"
