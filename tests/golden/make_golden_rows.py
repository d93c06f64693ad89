"""Reference outputs for the row-subset cases of ``row_cases.py``.

Runs the Kunlunxin-FFT reference itself (its Triton kernels on the CPU
through ``TRITON_INTERPRET=1``, set up exactly as ``make_golden.py`` does) on
the first rows of each BASELINE configuration the main golden set does not
reach, and writes ``reference_rows.npz`` (sampled output values per case) and
``reference_rows.json`` (the cases, the reference function used and its
float64 error).  The interpreter needs minutes for the 2^19 / 2^20 rows.

Usage::

    python tests/golden/make_golden_rows.py --ref PATH_TO_REFERENCE [--only LABEL ...]
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import row_cases  # noqa: E402
from make_golden import _setup_reference  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BFFT_REFERENCE_ROOT"),
                    help="reference tree (default: $BFFT_REFERENCE_ROOT); required")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference tree with --ref or BFFT_REFERENCE_ROOT")

    runner = _setup_reference(args.ref)
    import torch
    from src.xpu.config import DeviceProfile
    from src.xpu.entry import execute_fft_plan, plan_fft

    ph = DeviceProfile.load().hash()
    env = "6b50bd316032c0fe"  # the reference table's bound fingerprint

    # a table plan of each real-flow kind, re-targeted at the case's shape
    # (execute_fft_plan reads n, batch and params from the plan)
    base = {
        "c2c": plan_fft("dit", 1024, batch=16, profile_hash=ph, env_hash=env),
        "r2c": plan_fft("dit", 4096, batch=16, profile_hash=ph, env_hash=env, transform_type="r2c"),
        "c2r": plan_fft("dit", 4096, batch=16, profile_hash=ph, env_hash=env, transform_type="c2r"),
    }

    npz_path = os.path.join(args.out, "reference_rows.npz")
    json_path = os.path.join(args.out, "reference_rows.json")
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    if args.only and os.path.exists(npz_path):
        arrays = dict(np.load(npz_path))
        with open(json_path) as f:
            meta = json.load(f)["cases"]

    for case in row_cases.CASES:
        lab = case["label"]
        if args.only and lab not in args.only:
            continue
        x = row_cases.case_input(case)
        t = torch.from_numpy(x)
        t0 = time.time()
        if case["ref"] == "plan":
            params = dict(case["params"], batch=case["rows"])
            p = dataclasses.replace(base[case["tt"]], n=case["n"], batch=case["rows"], executed=case["executed"],
                                    params=params, transform_direction=case["td"])
            y = execute_fft_plan(p, t)
            how = {"entry": "execute_fft_plan", "executed": p.executed, "params": p.params,
                   "transform_type": p.transform_type, "transform_direction": p.transform_direction,
                   "norm": p.norm}
        else:
            fn = getattr(runner, case["ref"])
            y = fn(t, block=256, **case["knobs"])
            how = {"entry": case["ref"], "knobs": case["knobs"]}
        y = y.numpy()
        secs = time.time() - t0
        # float64 error of the reference's output (context for the fixture)
        x64 = x.astype(np.float64 if case["tt"] == "r2c" else np.complex128)
        if case["tt"] == "c2c":
            ref64 = np.fft.fft(x64, axis=-1) if case["td"] == "forward" else np.fft.ifft(x64, axis=-1)
        elif case["tt"] == "r2c":
            ref64 = np.fft.rfft(x64, axis=-1)
        else:
            ref64 = np.fft.irfft(x64, n=case["n"], axis=-1)
        err = float(np.linalg.norm(y.astype(ref64.dtype) - ref64) / np.linalg.norm(ref64))
        pos = row_cases.sample_positions(case, y.shape)
        arrays[f"{lab}__pos"] = pos
        arrays[f"{lab}__out"] = y.reshape(-1)[pos]
        meta[lab] = {**{k: v for k, v in case.items()}, "reference": how, "out_shape": list(y.shape),
                     "out_dtype": str(y.dtype), "rel_l2_vs_float64": err, "seconds": round(secs, 1)}
        print(f"  {lab}: {how['entry']} out {y.shape} rel_l2 vs f64 {err:.2e} ({secs:.0f} s)", flush=True)

    np.savez_compressed(npz_path, **arrays)
    with open(json_path, "w") as f:
        json.dump({"samples_per_case": row_cases.SAMPLES, "cases": meta}, f, indent=1, sort_keys=True,
                  default=str)
    print("wrote", len(meta), "cases")


if __name__ == "__main__":
    main()
