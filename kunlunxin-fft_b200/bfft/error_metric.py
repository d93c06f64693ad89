"""Correctness metrics (reference: src/xpu/error_metric.py).

``max_rel_error`` is the reference's contract metric -- peak-normalised
component-wise deviation, ``inf`` for any non-finite value.  ``rel_l2`` is
the relative L2 error the B200 parity gates use (<= 2e-6 against the
reference's own implementation, <= 1e-6 against float64 numpy).
"""
from __future__ import annotations

import numpy as np


def max_rel_error(got, ref) -> float:
    g = np.asarray(got)
    r = np.asarray(ref)
    delta = np.maximum(np.abs(g.real - r.real), np.abs(g.imag - r.imag))
    scale = np.abs(r).max()
    if not np.isfinite(delta).all() or not np.isfinite(scale):
        return float("inf")
    return float(delta.max() / max(float(scale), 1e-12))


def rel_l2(got, ref) -> float:
    g = np.asarray(got).astype(np.complex128)
    r = np.asarray(ref).astype(np.complex128)
    if not (np.isfinite(g).all() and np.isfinite(r).all()):
        return float("inf")
    return float(np.linalg.norm(g - r) / max(float(np.linalg.norm(r)), 1e-300))


def rel_l2_per_transform(got, ref) -> float:
    """Worst relative L2 error over the rows of (B, N) arrays."""
    g = np.asarray(got).astype(np.complex128)
    r = np.asarray(ref).astype(np.complex128)
    g = g.reshape(1, -1) if g.ndim == 1 else g
    r = r.reshape(1, -1) if r.ndim == 1 else r
    if not (np.isfinite(g).all() and np.isfinite(r).all()):
        return float("inf")
    num = np.linalg.norm(g - r, axis=1)
    den = np.maximum(np.linalg.norm(r, axis=1), 1e-300)
    return float((num / den).max())
