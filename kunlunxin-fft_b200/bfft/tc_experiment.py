"""Tensor-core (3xTF32 tcgen05.mma) 16-point row DFT against the FP32 row path.

The reference computes a tile's DFT as a dense FP32 matrix product
(src/xpu/kernels.py:487-532, local_matrix_kernel).  bfft_tc_dft16_rows is that
product on the B200 tensor cores with the 3xTF32 split; the product path for
the same shape is the plan the table resolves for N = 16 (FP32 radix-16
butterflies, one CTA-resident pass).  This measures both on the same seeded
input:

  * error: relative L2 against float64 numpy on a sample of rows, forward
    and inverse (1/N scale);
  * time: CUDA-event device time of one launch over ``rows`` rows (inputs
    and outputs of 2 x rows x 128 bytes; at the default 2^20 rows the pair is
    256 MiB, past the 126 MB L2), median of interleaved trials, with the
    achieved HBM GB/s (read + write once).

Run: ``python -m bfft.tc_experiment [--rows R] [--trials T]`` with the package
directory on PYTHONPATH; prints one JSON object.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import _lib
from .config import DeviceProfile
from .entry import ExecutionPlan, native_plan_for, plan_fft
from .runner import execute_native, time_call_detailed

N = 16


def tc_rows(x: torch.Tensor, out: torch.Tensor, inverse: bool = False, scale: float = 1.0) -> torch.Tensor:
    """out[r] = DFT16(x[r]) (or the inverse, times scale) on the tensor cores."""
    rows = x.numel() // N
    dev = x.device.index or 0
    st = _lib.load().bfft_tc_dft16_rows(x.data_ptr(), out.data_ptr(), rows, 1 if inverse else 0, float(scale), dev,
                                        torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st, "bfft_tc_dft16_rows")
    return out


def product_plan(rows: int, transform_direction: str) -> ExecutionPlan:
    """The plan the public API resolves for (N = 16, batch = rows) on this
    device; where the table abstains, the local-fused core with tile = N (the
    table's choice for every measured small-N batch)."""
    p = plan_fft("dit", N, batch=rows, profile_hash=DeviceProfile.load().hash(),
                 transform_direction=transform_direction)
    if not p.fallback:
        return p
    return ExecutionPlan(n=N, batch=rows, direction="dit", precision="fp32", selection_source="table",
                         reason="explicit local-fused core (table abstained: " + p.reason + ")", fallback=False,
                         executed="fft_dit_matrix_batch" if rows > 1 else "fft_dit_matrix", block=256,
                         flow_id="local-fused-tile", flow_realization="matrix-resident",
                         processing_unit="dense-dot-fft64",
                         params={"tile": N, "rows": 1, "variant": "spread", "batch": rows},
                         transform_direction=transform_direction)


def rel_l2_f64(got: np.ndarray, x: np.ndarray, inverse: bool) -> float:
    x64 = x.astype(np.complex128)
    ref = np.fft.ifft(x64, axis=-1) if inverse else np.fft.fft(x64, axis=-1)
    g = got.astype(np.complex128)
    return float(np.linalg.norm(g - ref) / np.linalg.norm(ref))


def measure(rows: int = 1 << 20, trials: int = 30, sample_rows: int = 1 << 16, seed: int = 20260) -> dict:
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(seed)
    xh = (rng.standard_normal((rows, N)) + 1j * rng.standard_normal((rows, N))).astype(np.complex64)
    x = torch.from_numpy(xh).to(dev)
    y_tc = torch.empty_like(x)
    y_fp = torch.empty_like(x)
    plan = product_plan(rows, "forward")
    nplan = native_plan_for(plan, dev.index or 0)
    nplan_inv = native_plan_for(product_plan(rows, "inverse"), dev.index or 0)

    def fp32_rows(out, inverse=False):
        return execute_native(nplan_inv if inverse else nplan, x, out)

    s = sample_rows
    res = {"n": N, "rows": rows, "sample_rows": s, "seed": seed,
           "product_plan": {"executed": plan.executed, "tile": plan.params.get("tile"),
                            "source": plan.reason[:80], "launches": nplan.launches}}
    _lib.device_status(dev.index or 0, clear=True)
    for inverse in (False, True):
        tc_rows(x, y_tc, inverse, 1.0 / N if inverse else 1.0)
        fp32_rows(y_fp, inverse)
        torch.cuda.synchronize()
        tag = "inverse" if inverse else "forward"
        got_tc = y_tc[:s].cpu().numpy()
        got_fp = y_fp[:s].cpu().numpy()
        res[f"rel_l2_vs_f64_{tag}"] = {"tc_3xtf32": rel_l2_f64(got_tc, xh[:s], inverse),
                                       "fp32_rows": rel_l2_f64(got_fp, xh[:s], inverse)}
        # largest element-wise error relative to the row's norm
        x64 = xh[:s].astype(np.complex128)
        ref = np.fft.ifft(x64, axis=-1) if inverse else np.fft.fft(x64, axis=-1)
        rn = np.linalg.norm(ref, axis=-1, keepdims=True)
        res[f"max_rowrel_{tag}"] = {"tc_3xtf32": float(np.max(np.abs(got_tc - ref) / rn)),
                                    "fp32_rows": float(np.max(np.abs(got_fp - ref) / rn))}
    bytes_moved = 2 * rows * N * 8
    t_tc = time_call_detailed(lambda: tc_rows(x, y_tc), warmup=5, trials=trials, seed=1)["kernel_ms"]["median"]
    t_fp = time_call_detailed(lambda: fp32_rows(y_fp), warmup=5, trials=trials, seed=2)["kernel_ms"]["median"]
    res["ms"] = {"tc_3xtf32": t_tc, "fp32_rows": t_fp}
    res["hbm_gbs"] = {"tc_3xtf32": bytes_moved / t_tc / 1e6, "fp32_rows": bytes_moved / t_fp / 1e6}
    res["device_status"] = _lib.device_status(dev.index or 0)
    return res


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rows", type=int, default=1 << 20)
    ap.add_argument("--trials", type=int, default=30)
    ap.add_argument("--sample-rows", type=int, default=1 << 16)
    a = ap.parse_args()
    print(json.dumps(measure(a.rows, a.trials, min(a.sample_rows, a.rows))))


if __name__ == "__main__":
    main()
