"""Phase markers of execute_fft_plan (reference: src/xpu/ledger.py:64-148).

``phase(name)`` is a no-op unless a :class:`PhaseLedger` is active in the
current context; then each phase is bracketed by ``torch.cuda.synchronize()``
and its wall time recorded, and an NVTX range with the same name is pushed so
the phases line up with profiler timelines.
"""
from __future__ import annotations

import contextlib
import contextvars
import time

_ACTIVE: contextvars.ContextVar = contextvars.ContextVar("bfft_phase_ledger", default=None)


class PhaseLedger:
    """Collects (phase, milliseconds) pairs while active."""

    def __init__(self):
        self.rows: list[tuple[str, float]] = []
        self._token = None

    def __enter__(self):
        self._token = _ACTIVE.set(self)
        return self

    def __exit__(self, *exc):
        _ACTIVE.reset(self._token)
        return False

    def totals(self) -> dict:
        out: dict = {}
        for name, ms in self.rows:
            out[name] = out.get(name, 0.0) + ms
        return out


@contextlib.contextmanager
def phase(name: str):
    ledger = _ACTIVE.get()
    if ledger is None:
        yield
        return
    import torch

    nvtx = getattr(torch.cuda, "nvtx", None)
    torch.cuda.synchronize()
    if nvtx is not None:
        nvtx.range_push(name)
    t0 = time.perf_counter()
    try:
        yield
    finally:
        torch.cuda.synchronize()
        ledger.rows.append((name, (time.perf_counter() - t0) * 1e3))
        if nvtx is not None:
            nvtx.range_pop()
