"""Generate golden vectors by running the Kunlunxin-FFT reference itself.

Run in a container that has the read-only reference tree (``--ref``, or the
``BFFT_REFERENCE_ROOT`` environment variable) and Triton; the reference's Triton kernels execute on the
CPU through ``TRITON_INTERPRET=1``.  The output, ``reference_vectors.npz`` plus
``reference_plans.json``, is committed next to this script so the GPU box
(which has no reference tree) and the CPU test suite can use it.

Nothing here is imported by the product.  The reference is called through its
own public functions (``src/xpu/entry.py``, ``src/xpu/runner.py``,
``src/xpu/adapter_hybrid.py``); the only patches make its device guards accept
CPU tensors (its validation requires ``device.type == 'cuda'``).

Usage::

    python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE]
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# Synthetic selector table used to record the reference's plan semantics
# (tiers, fallbacks, reasons).  Written for this test; not reference data.
SYNTH_TABLE = {
    "schema_version": 2,
    "device": "synthetic",
    "profile_hash": "p-synth-0001",
    "env_hash": "e-synth-0001",
    "env": {"device_model": 1, "multiprocessor_count": 2, "max_shared_mem": 1024},
    "precision": "fp32",
    "guard_pct": 2.0,
    "entries": [
        {"N": 1024, "batch": 1, "direction": "dit", "block": 256,
         "incumbent_block": 512, "flow_id": "local-fused-tile",
         "flow_realization": "matrix-resident",
         "processing_unit": "dense-dot-fft64",
         "params": {"tile": 64, "rows": 8},
         "reason": "synthetic legacy winner m2"},
        {"N": 1024, "batch": 16, "direction": "dit", "block": 512,
         "flow_id": "local-fused-tile", "flow_realization": "matrix-resident",
         "processing_unit": "dense-dot-fft64",
         "params": {"tile": 128, "rows": 8, "variant": "spread", "batch": 16},
         "transform_type": "c2c", "transform_direction": "forward",
         "normalization": "backward", "reason": "synthetic semantic winner"},
        {"N": 1024, "batch": 16, "direction": "dit", "block": 1024,
         "flow_id": "batch-spread", "flow_realization": "global-stage",
         "processing_unit": "radix4-scalar",
         "params": {"variant": "spread", "batch": 16},
         "transform_type": "c2c", "transform_direction": "inverse",
         "normalization": "backward", "executed": "fft_dif_radix4_batch",
         "reason": "synthetic inverse winner"},
        {"N": 256, "batch": 1, "direction": "dit", "block": 128,
         "flow_id": "local-fused-tile", "flow_realization": "fused-inplace",
         "processing_unit": "radix2-scalar", "params": {"tile": 64},
         "reason": "synthetic m1"},
        {"N": 256, "batch": 4, "direction": "dit", "block": 128,
         "flow_id": "local-fused-tile", "flow_realization": "fused-inplace",
         "processing_unit": "radix2-scalar", "params": {"tile": 64, "batch": 4,
                                                         "variant": "spread"},
         "reason": "synthetic batched m1 (no lowering)"},
        {"N": 4096, "batch": 16, "direction": "dit", "block": 1024,
         "flow_id": "dedicated-r2c-pack-v1",
         "flow_realization": "matrix-resident",
         "processing_unit": "dense-dot-fft64",
         "params": {"real_flow": "dedicated-r2c-pack-v1", "tile": 64,
                    "rows": 8, "variant": "spread", "batch": 16},
         "transform_type": "r2c", "transform_direction": "forward",
         "normalization": "backward", "executed": "fft_dif_matrix_batch",
         "reason": "synthetic r2c dedicated"},
        {"N": 4096, "batch": 16, "direction": "dit", "block": 1024,
         "flow_id": "dedicated-c2r-hermitian-v1",
         "flow_realization": "matrix-resident",
         "processing_unit": "dense-dot-fft64",
         "params": {"real_flow": "dedicated-c2r-hermitian-v1", "tile": 64,
                    "rows": 8, "variant": "spread", "batch": 16},
         "transform_type": "c2r", "transform_direction": "inverse",
         "normalization": "backward", "executed": "fft_dit_matrix_batch",
         "reason": "synthetic c2r dedicated"},
        {"N": 2048, "batch": 1, "direction": "dif", "block": 512,
         "flow_id": "baseline-global-stage", "flow_realization": "global-stage",
         "processing_unit": "radix4-scalar", "params": {},
         "reason": "synthetic m5 dif"},
    ],
    "previous_fallbacks": [
        {"N": 1024, "batch": 16, "direction": "dit", "block": 256,
         "flow_id": "local-fused-tile", "flow_realization": "matrix-resident",
         "processing_unit": "dense-dot-fft64",
         "params": {"tile": 64, "rows": 4, "variant": "spread", "batch": 16},
         "transform_type": "c2c", "transform_direction": "forward",
         "normalization": "ortho", "reason": "synthetic fallback cell"},
    ],
}

# (label, kwargs for plan_fft) recorded against SYNTH_TABLE.
PLAN_QUERIES = [
    ("legacy-hit", dict(direction="dit", n=1024, batch=1)),
    ("semantic-hit", dict(direction="dit", n=1024, batch=16)),
    ("semantic-inverse-executed", dict(direction="dit", n=1024, batch=16,
                                       transform_direction="inverse")),
    ("previous-fallback", dict(direction="dit", n=1024, batch=16, norm="ortho")),
    ("semantic-miss-abstain", dict(direction="dit", n=1024, batch=16,
                                   norm="forward")),
    ("legacy-inverse", dict(direction="dit", n=1024, batch=1,
                            transform_direction="inverse")),
    ("m1-hit", dict(direction="dit", n=256, batch=1)),
    ("m1-batched-undispatchable", dict(direction="dit", n=256, batch=4)),
    ("unknown-n", dict(direction="dit", n=8192, batch=1)),
    ("unknown-n-batched", dict(direction="dif", n=8192, batch=4)),
    ("r2c-dedicated", dict(direction="dit", n=4096, batch=16,
                           transform_type="r2c")),
    ("c2r-dedicated", dict(direction="dit", n=4096, batch=16,
                           transform_type="c2r")),
    ("r2c-legacy-compat", dict(direction="dit", n=1024, batch=1,
                               transform_type="r2c")),
    ("c2r-abstain-compat", dict(direction="dit", n=512, batch=2,
                                transform_type="c2r")),
    ("m5-dif", dict(direction="dif", n=2048, batch=1)),
    ("profile-none", dict(direction="dit", n=1024, batch=1, profile_hash=None)),
    ("profile-mismatch", dict(direction="dit", n=1024, batch=1,
                              profile_hash="p-other")),
    ("env-none", dict(direction="dit", n=1024, batch=1, env_hash=None)),
    ("env-mismatch", dict(direction="dit", n=1024, batch=1, env_hash="e-other")),
    ("precision-table-mismatch-dif", dict(direction="dif", n=1024, batch=1)),
]


def _setup_reference(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch  # noqa: F401
    import src.xpu.context as ctx
    import src.xpu.runner as runner

    ctx.device_ready = lambda: True
    runner.device_ready = lambda: True
    runner.xpu_context = lambda *a, **k: contextlib.nullcontext()

    def _validate_input(x, name="x", *, allow_n=None, block=None,
                        require_complex=True):
        assert x.dim() == 1 and x.is_contiguous(), name

    def _validate_batch(x, block, variant):
        if variant not in ("spread", "folded"):
            raise ValueError(variant)
        b, n = x.shape
        return b, n

    def _validate_half(x, n, bins, name):
        assert x.shape[-1] == bins, (name, x.shape, bins)

    runner.validate_input = _validate_input
    runner._validate_batch_input = _validate_batch
    runner._validate_real_half = _validate_half
    return runner


def _cplx(rng, shape):
    re = rng.standard_normal(shape).astype(np.float32)
    im = rng.standard_normal(shape).astype(np.float32)
    return (re + 1j * im).astype(np.complex64)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BFFT_REFERENCE_ROOT"),
                    help="reference tree (default: $BFFT_REFERENCE_ROOT); required")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference tree with --ref or BFFT_REFERENCE_ROOT")

    runner = _setup_reference(args.ref)
    import torch
    import triton
    import triton.language as tl
    from src.xpu import adapter_hybrid, kernels
    from src.xpu.config import DeviceProfile
    from src.xpu.entry import execute_fft_plan, plan_fft

    out: dict[str, np.ndarray] = {}
    cases: list[dict] = []
    # the interpreter resolves names through this module's globals
    globals()["kernels"] = kernels
    globals()["tl"] = tl

    # ---- index maps, straight from the reference's jit helpers ---------
    @triton.jit
    def _index_kernel(OUT, N, BITS: tl.constexpr, KIND: tl.constexpr,
                      BLOCK: tl.constexpr):
        off = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        mask = off < N
        if KIND == 0:
            v = kernels._bit_reverse(off, BITS)
        elif KIND == 1:
            v = kernels._dit_digit_reverse(off, BITS)
        else:
            v = kernels._dif_digit_reverse(off, BITS)
        tl.store(OUT + off, v, mask=mask)

    for kind, name in ((0, "bitrev"), (1, "dit_digrev"), (2, "dif_digrev")):
        for bits in range(1, 13):
            n = 1 << bits
            o = torch.zeros(n, dtype=torch.int32)
            _index_kernel[(triton.cdiv(n, 1024),)](o, n, BITS=bits, KIND=kind,
                                                   BLOCK=1024)
            out[f"idx_{name}_{bits}"] = o.numpy().astype(np.uint32)

    # bit_reverse_permute on an index-valued input (tests/test_fft.py:77-95 style)
    for n in (8, 64, 1024):
        x = torch.arange(n, dtype=torch.float32).to(torch.complex64)
        out[f"bitrev_permute_{n}"] = runner.bit_reverse_permute(x).numpy()

    def add(label, fn, x, **meta):
        y = fn(torch.from_numpy(x))
        y = y.numpy() if hasattr(y, "numpy") else np.asarray(y)
        out[f"{label}__in"] = x
        out[f"{label}__out"] = y
        cases.append({"label": label, **meta})
        print(f"  {label}: in {x.shape} {x.dtype} -> out {y.shape}", flush=True)

    rng = np.random.default_rng(20261201)

    # ---- per-runner outputs --------------------------------------------
    R = runner
    add("fft_dit_256", lambda t: R.fft_dit(t, block=64), _cplx(rng, 256),
        runner="fft_dit", n=256, batch=1)
    add("fft_dif_256", lambda t: R.fft_dif(t, block=64), _cplx(rng, 256),
        runner="fft_dif", n=256, batch=1)
    add("fft_dit_2", lambda t: R.fft_dit(t, block=64), _cplx(rng, 2),
        runner="fft_dit", n=2, batch=1)
    add("fft_dit_batch_spread_128x4",
        lambda t: R.fft_dit_batch(t, block=64, variant="spread"),
        _cplx(rng, (4, 128)), runner="fft_dit_batch", n=128, batch=4,
        variant="spread")
    add("fft_dit_batch_folded_128x4",
        lambda t: R.fft_dit_batch(t, block=64, variant="folded"),
        _cplx(rng, (4, 128)), runner="fft_dit_batch", n=128, batch=4,
        variant="folded")
    add("fft_dif_batch_folded_64x8",
        lambda t: R.fft_dif_batch(t, block=64, variant="folded"),
        _cplx(rng, (8, 64)), runner="fft_dif_batch", n=64, batch=8,
        variant="folded")
    for n in (4, 8, 512, 1024):
        add(f"fft_dit_radix4_{n}", lambda t: R.fft_dit_radix4(t, block=64),
            _cplx(rng, n), runner="fft_dit_radix4", n=n, batch=1)
        add(f"fft_dif_radix4_{n}", lambda t: R.fft_dif_radix4(t, block=64),
            _cplx(rng, n), runner="fft_dif_radix4", n=n, batch=1)
    for n in (512, 2048):
        add(f"fft_dit_radix4_batch_{n}x4",
            lambda t: R.fft_dit_radix4_batch(t, block=256),
            _cplx(rng, (4, n)), runner="fft_dit_radix4_batch", n=n, batch=4)
        add(f"fft_dif_radix4_batch_{n}x4",
            lambda t: R.fft_dif_radix4_batch(t, block=256),
            _cplx(rng, (4, n)), runner="fft_dif_radix4_batch", n=n, batch=4)
    add("fft_dit_fused_256_t64", lambda t: R.fft_dit_fused(t, block=64, tile=64),
        _cplx(rng, 256), runner="fft_dit_fused", n=256, batch=1, tile=64)
    add("fft_dit_fused_32_t64", lambda t: R.fft_dit_fused(t, block=64, tile=64),
        _cplx(rng, 32), runner="fft_dit_fused", n=32, batch=1, tile=64)
    add("fft_dit_matrix_512_t64",
        lambda t: R.fft_dit_matrix(t, block=128, tile=64, rows=8),
        _cplx(rng, 512), runner="fft_dit_matrix", n=512, batch=1, tile=64, rows=8)
    add("fft_dif_matrix_512_t32",
        lambda t: R.fft_dif_matrix(t, block=128, tile=32, rows=4),
        _cplx(rng, 512), runner="fft_dif_matrix", n=512, batch=1, tile=32, rows=4)
    add("fft_dit_matrix_batch_1024x4_t128",
        lambda t: R.fft_dit_matrix_batch(t, block=256, tile=128, rows=8),
        _cplx(rng, (4, 1024)), runner="fft_dit_matrix_batch", n=1024, batch=4,
        tile=128, rows=8)
    add("fft_dif_matrix_batch_1024x4_t64",
        lambda t: R.fft_dif_matrix_batch(t, block=256, tile=64, rows=8),
        _cplx(rng, (4, 1024)), runner="fft_dif_matrix_batch", n=1024, batch=4,
        tile=64, rows=8)
    add("fft_dit_grouped_1024_t8",
        lambda t: R.fft_dit_grouped(t, block=256, tile=8, rows=8, glog=2,
                                    maxp=4096, cells=1),
        _cplx(rng, 1024), runner="fft_dit_grouped", n=1024, batch=1, tile=8,
        rows=8, glog=2, maxp=4096, cells=1)
    add("fft_dif_grouped_1024_t8",
        lambda t: R.fft_dif_grouped(t, block=256, tile=8, rows=8, glog=2,
                                    maxp=4096, cells=1),
        _cplx(rng, 1024), runner="fft_dif_grouped", n=1024, batch=1, tile=8,
        rows=8, glog=2, maxp=4096, cells=1)

    # ---- hybrid 4-step with the reference's own (triton) local core ----
    hp = adapter_hybrid.plan_hybrid(2048, 16, tile=64, core="triton")
    add("run_hybrid_2048x16_t64", lambda t: adapter_hybrid.run_hybrid(t, hp),
        _cplx(rng, (16, 2048)), runner="run_hybrid", n=2048, batch=16, tile=64)
    hp2 = adapter_hybrid.plan_hybrid(1024, 2, tile=32, core="triton")
    add("run_hybrid_1024x2_t32", lambda t: adapter_hybrid.run_hybrid(t, hp2),
        _cplx(rng, (2, 1024)), runner="run_hybrid", n=1024, batch=2, tile=32)

    # ---- real-transform epilogues (device kernels) ----------------------
    for n, b in ((64, 3), (1024, 2)):
        add(f"r2c_stitch_{n}x{b}", lambda t, n=n: R.r2c_stitch(t, n, scale=0.5,
                                                               block=64),
            _cplx(rng, (b, n // 2)), runner="r2c_stitch", n=n, batch=b,
            scale=0.5)
        add(f"c2r_pre_{n}x{b}", lambda t, n=n: R.c2r_pre(t, n, block=64),
            _cplx(rng, (b, n // 2 + 1)), runner="c2r_pre", n=n, batch=b)
        add(f"c2r_unpack_{n}x{b}", lambda t, n=n: R.c2r_unpack(t, n, scale=0.25,
                                                               block=64),
            _cplx(rng, (b, n // 2)), runner="c2r_unpack", n=n, batch=b,
            scale=0.25)

    # ---- full plans through the public API (P800 profile + table) ------
    ph = DeviceProfile.load().hash()
    env = "6b50bd316032c0fe"   # the reference table's bound fingerprint

    def plan_case(label, n, b, x, **kw):
        p = plan_fft(kw.pop("direction", "dit"), n, batch=b, profile_hash=ph,
                     env_hash=env, **kw)
        add(label, lambda t: execute_fft_plan(p, t), x, plan=dict(
            executed=p.executed, fallback=p.fallback,
            selection_source=p.selection_source, params=p.params,
            transform_type=p.transform_type,
            transform_direction=p.transform_direction, norm=p.norm),
            n=n, batch=b)

    plan_case("plan_c2c_fwd_2048x1", 2048, 1, _cplx(rng, 2048))
    plan_case("plan_c2c_fwd_1024x16", 1024, 16, _cplx(rng, (16, 1024)))
    plan_case("plan_c2c_inv_1024x16", 1024, 16, _cplx(rng, (16, 1024)),
              transform_direction="inverse")
    plan_case("plan_c2c_inv_2048x16", 2048, 16, _cplx(rng, (16, 2048)),
              transform_direction="inverse")
    plan_case("plan_c2c_fwd_65536x1", 65536, 1, _cplx(rng, 65536))
    for norm in ("none", "forward", "backward", "ortho"):
        for tdir in ("forward", "inverse"):
            plan_case(f"plan_c2c_{tdir}_{norm}_256x4", 256, 4,
                      _cplx(rng, (4, 256)), transform_direction=tdir, norm=norm)
    xr = rng.standard_normal((16, 4096)).astype(np.float32)
    plan_case("plan_r2c_4096x16", 4096, 16, xr, transform_type="r2c")
    xh = np.fft.rfft(rng.standard_normal((16, 4096))).astype(np.complex64)
    plan_case("plan_c2r_4096x16", 4096, 16, xh, transform_type="c2r")
    for norm in ("forward", "ortho"):
        plan_case(f"plan_r2c_{norm}_256x1", 256, 1,
                  rng.standard_normal(256).astype(np.float32),
                  transform_type="r2c", norm=norm)
        plan_case(f"plan_c2r_{norm}_256x1", 256, 1,
                  np.fft.rfft(rng.standard_normal(256)).astype(np.complex64),
                  transform_type="c2r", norm=norm)

    # ---- known-answer signals (tests/test_fft.py:196-211) ---------------
    imp = np.zeros(256, np.complex64)
    imp[0] = 1
    tone = np.exp(2j * np.pi * 5 * np.arange(256) / 256).astype(np.complex64)
    const = np.full(256, 3 + 4j, np.complex64)
    for name, sig in (("impulse", imp), ("tone5", tone), ("const34", const)):
        add(f"kat_{name}_256", lambda t: R.fft_dit(t, block=64), sig,
            runner="fft_dit", n=256, batch=1)

    # ---- plan semantics against a synthetic table -----------------------
    plans = {}
    for label, q in PLAN_QUERIES:
        q = dict(q)
        q.setdefault("profile_hash", SYNTH_TABLE["profile_hash"])
        q.setdefault("env_hash", SYNTH_TABLE["env_hash"])
        try:
            p = plan_fft(table=SYNTH_TABLE, **q)
            plans[label] = {"query": q, "plan": {k: v for k, v in p.__dict__.items()}}
        except Exception as e:  # noqa: BLE001 - record the raised type/message
            plans[label] = {"query": q, "raises": type(e).__name__, "msg": str(e)}
    bad_semantics = [
        dict(direction="fft", n=256), dict(direction="dit", n=256, precision="fp16"),
        dict(direction="dit", n=256, transform_type="dct"),
        dict(direction="dit", n=256, transform_direction="sideways"),
        dict(direction="dit", n=256, norm="unit"),
        dict(direction="dit", n=256, transform_type="r2c",
             transform_direction="inverse"),
        dict(direction="dit", n=256, transform_type="c2r",
             transform_direction="forward"),
    ]
    for i, q in enumerate(bad_semantics):
        try:
            plan_fft(table=SYNTH_TABLE, profile_hash="p-synth-0001",
                     env_hash="e-synth-0001", **q)
            plans[f"bad-{i}"] = {"query": q, "raises": None}
        except Exception as e:  # noqa: BLE001
            plans[f"bad-{i}"] = {"query": q, "raises": type(e).__name__,
                                 "msg": str(e)}

    np.savez_compressed(os.path.join(args.out, "reference_vectors.npz"), **out)
    with open(os.path.join(args.out, "reference_plans.json"), "w") as f:
        json.dump({"synthetic_table": SYNTH_TABLE, "plans": plans,
                   "cases": cases}, f, indent=1, sort_keys=True, default=str)
    print("wrote", len(out), "arrays and", len(plans), "plan records")


if __name__ == "__main__":
    main()
