"""Plans executed on host (CPU) arrays with overlapped PCIe copies.

The reference's operator API takes device tensors.  ``execute_fft_plan_host``
runs a resolved plan on a host tensor: the batch is split into chunks and the
copy in of chunk k+1, the transform of chunk k and the copy out of chunk k-1
overlap on three streams inside libbfft (``bfft_stream_*``), so a host-to-host
transform costs about one PCIe direction instead of both plus the transform.
No counterpart in the reference; there is no CPU fallback.
"""
from __future__ import annotations

import threading
from collections import OrderedDict

import torch

from . import _lib
from .entry import ExecutionPlan, _check_plan_input, _runner_knobs

_CHUNK_TARGET_BYTES = 64 << 20
_STREAM_PLANS: "OrderedDict[tuple, _lib.NativeStreamPlan]" = OrderedDict()
_LOCK = threading.Lock()
_MAX = 16


def default_chunks(plan: ExecutionPlan) -> int:
    """Power-of-two chunk count dividing the batch, chunks of about 64 MiB."""
    row_bytes = 8 * plan.n
    want = max(1, (plan.batch * row_bytes) // _CHUNK_TARGET_BYTES)
    c = 1
    while c * 2 <= want and plan.batch % (c * 2) == 0:
        c *= 2
    return c


def stream_plan(plan: ExecutionPlan, chunks: int, device: int) -> _lib.NativeStreamPlan:
    if plan.executed not in _lib.RUNNER_IDS:
        raise ValueError(f"plan runner {plan.executed!r} has no native lowering")
    if chunks < 1 or plan.batch % chunks:
        raise ValueError(f"chunks={chunks} must divide the batch {plan.batch}")
    knobs = _runner_knobs(plan)
    variant = knobs.pop("variant", "spread")
    real_flow = bool((plan.params or {}).get("real_flow")) and plan.transform_type != "c2c"
    key = (plan.executed, plan.direction, plan.n, plan.batch, plan.transform_type, plan.transform_direction,
           plan.norm, real_flow, variant, tuple(sorted(knobs.items())), chunks, device)
    with _LOCK:
        sp = _STREAM_PLANS.get(key)
        if sp is not None:
            _STREAM_PLANS.move_to_end(key)
            return sp
    desc = _lib.make_desc(plan.executed, plan.direction, plan.n, plan.batch // chunks,
                          transform_type=plan.transform_type, transform_direction=plan.transform_direction,
                          norm=plan.norm, real_flow=real_flow, variant=variant, device=device, **knobs)
    with torch.cuda.device(device):
        sp = _lib.NativeStreamPlan(desc, chunks)
    with _LOCK:
        _STREAM_PLANS[key] = sp
        while len(_STREAM_PLANS) > _MAX:
            _STREAM_PLANS.popitem(last=False)
    return sp


def execute_fft_plan_host(plan: ExecutionPlan, x: torch.Tensor, out: torch.Tensor | None = None, *,
                          chunks: int | None = None, device: int | None = None) -> torch.Tensor:
    """Execute ``plan`` on a host tensor and return a host tensor.

    ``x`` has the plan's input shape and dtype on the CPU (page-locked for the
    copies to overlap); the result is written to ``out`` (allocated pinned when
    omitted).  Enqueued on the current stream of ``device``; the call returns
    once the result is in host memory."""
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
    if x.device.type != "cpu":
        raise ValueError(f"x must be a host (CPU) tensor, got device={x.device}")
    _check_plan_input(plan, tuple(x.shape), str(x.dtype).split(".")[-1])
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    dev = torch.cuda.current_device() if device is None else int(device)
    sp = stream_plan(plan, chunks or default_chunks(plan), dev)
    lead = tuple(x.shape[:-1])
    if plan.transform_type == "r2c":
        shape, dtype = (*lead, plan.n // 2 + 1), torch.complex64
    elif plan.transform_type == "c2r":
        shape, dtype = (*lead, plan.n), torch.float32
    else:
        shape, dtype = tuple(x.shape), torch.complex64
    if out is None:
        out = torch.empty(shape, dtype=dtype, pin_memory=True)
    elif tuple(out.shape) != shape or out.dtype != dtype or out.device.type != "cpu" or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous host tensor {shape} {dtype}")
    stream = torch.cuda.current_stream(dev)
    sp.execute(x.data_ptr(), out.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    return out
