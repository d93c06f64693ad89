"""4-step (hybrid) decomposition N = T * R (reference: src/xpu/adapter_hybrid.py).

DIT, natural order in and out.  With ``tile`` = R and ``t2 = N / tile``::

    blocks[m0, m1] = x[m1 * tile + m0]            (gather, a strided view)
    C[m0, k_t]     = FFT_t2 over m1               (first sub-FFT pass)
    G[k_t, m0]     = C[m0, k_t] * W_N^{k_t m0}    (twiddle)
    X[k_r t2 + k_t] = FFT_tile over m0 of G[k_t]   (second pass, transposed store)

The reference materialises the gather, the twiddled grid and the output
transpose as separate tensors around a vendor or Triton core.  On B200 the
whole flow is two CTA-resident passes of libbfft: the gather is the first
pass's strided load, the twiddle its fused epilogue, the transpose the second
pass's store; the plan owns nothing but the native plan handle.
"""
from __future__ import annotations

from dataclasses import dataclass, field

CORES = ("b200-pass", "triton")


@dataclass
class HybridPlan:
    """Decomposition plan; ``core`` names the local sub-FFT core."""

    n: int
    batch: int
    tile: int
    direction: str = "dit"
    core: str = "b200-pass"
    stage2_len: int = field(init=False)

    def __post_init__(self):
        if self.direction != "dit":
            raise ValueError("the hybrid decomposition is DIT only")
        if (self.n & (self.n - 1)) or (self.tile & (self.tile - 1)) or self.n <= 0 or self.tile <= 0:
            raise ValueError("N and tile must be powers of two")
        if self.n % self.tile:
            raise ValueError(f"tile {self.tile} must divide N={self.n}")
        if self.core == "vendor":
            raise ValueError("core 'vendor' (a vendor whole-transform FFT) is not used on B200; "
                             "the local core is this library's pass kernel ('b200-pass')")
        if self.core not in CORES:
            raise ValueError(f"unknown core {self.core!r}")
        self.stage2_len = self.n // self.tile


def plan_hybrid(n: int, batch: int, tile: int = 64, core: str = "b200-pass") -> HybridPlan:
    return HybridPlan(n=n, batch=batch, tile=tile, core=core)


def run_hybrid(x, plan: HybridPlan):
    """Execute the 4-step flow on (B, N) complex64 (B = plan.batch); fresh output."""
    import torch

    from .runner import _device_index, execute_native, native_plan

    if not isinstance(x, torch.Tensor):
        raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != torch.complex64:
        raise TypeError(f"x must be complex64, got {x.dtype}")
    if x.dim() != 2 or tuple(x.shape) != (plan.batch, plan.n):
        raise ValueError(f"x must have shape ({plan.batch}, {plan.n}), got {tuple(x.shape)}")
    if x.device.type != "cuda" or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor")
    native = native_plan("run_hybrid", "dit", plan.n, plan.batch, _device_index(x), tile=plan.tile,
                         block=256)
    return execute_native(native, x, torch.empty_like(x))


def plan_ledger(plan: HybridPlan) -> dict:
    """Analytic accounting of one plan (reference adapter_hybrid.py:273-316):
    HBM passes, bytes and launches of the B200 flow."""
    elem = 8
    passes = int(plan.stage2_len > 1) + int(plan.tile > 1)
    return {
        "core": plan.core,
        "core_calls": {"stage1": plan.batch * plan.tile, "stage1_len": plan.stage2_len,
                       "stage2": plan.batch * plan.stage2_len, "stage2_len": plan.tile},
        "core_launches_est": passes,
        "materialized_boundaries": [{"op": "pass-1 store (twiddled columns)",
                                     "bytes_est": plan.batch * plan.n * elem}] if passes == 2 else [],
        "gm_bytes_framework_est": passes * 2 * plan.batch * plan.n * elem,
        "sync_points_per_timed_call": 0,
        "element_bytes_assumed": elem,
        "twiddle_and_row_tables": "plan-owned device tables (float64 rounded once)",
        "buffers": "caller workspace; output is fresh per call",
    }
