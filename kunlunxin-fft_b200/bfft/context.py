"""CUDA device guard (reference: src/xpu/context.py).

The reference wraps every launch in ``xpu_context`` because XPU launches
outside it silently do nothing.  On B200 the guard makes the tensor's device
current for the call (library calls also carry the device explicitly);
``xpu_context`` is kept as the API name.
"""
from __future__ import annotations

import contextlib


def device_ready() -> bool:
    """True when torch sees at least one CUDA device."""
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:  # noqa: BLE001
        return False


@contextlib.contextmanager
def xpu_context(device_index: int = 0):
    """Make ``device_index`` the current CUDA device for the block."""
    if not device_ready():
        raise RuntimeError("CUDA device stack not available; refusing to launch")
    import torch

    with torch.cuda.device(device_index):
        yield


cuda_context = xpu_context
