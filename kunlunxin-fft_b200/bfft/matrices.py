"""Host-side (numpy) descriptions of the local group and the tail partition.

Reference: src/xpu/matrices.py.  ``local_matrix`` is the linear map of the
first log2(tile) DIT stages on a bit-reversed tile (or the last log2(tile) DIF
stages), built by pushing unit vectors through the radix-2 stages; it depends
only on the tile.  On B200 the local group runs as a CTA-resident FFT pass,
so the matrix is kept as a host-side specification (tests use it to pin the
pass against the stage definition), not as device data.  ``tail_groups`` is
the reference's partition of the tail stages into execution groups, which the
M3 flow of libbfft applies identically (csrc/bfft_api.cu ``tail_groups``).
"""
from __future__ import annotations

import numpy as np


def _log2_exact(n: int) -> int:
    if n <= 0 or (n & (n - 1)):
        raise ValueError(f"expected a power of two, got {n}")
    return n.bit_length() - 1


def _stage(v: np.ndarray, half: int, direction: str) -> np.ndarray:
    """One radix-2 stage of half-span ``half`` on a vector (twiddle
    exp(-2j pi j / (2 half)), N-independent)."""
    w = np.exp(-2j * np.pi * np.arange(half) / (2 * half))
    blk = v.reshape(-1, 2 * half)
    lo, hi = blk[:, :half], blk[:, half:]
    if direction == "dit":
        hi = hi * w
        return np.concatenate((lo + hi, lo - hi), axis=1).reshape(v.shape)
    return np.concatenate((lo + hi, (lo - hi) * w), axis=1).reshape(v.shape)


def local_matrix(tile: int, direction: str = "dit") -> np.ndarray:
    """complex128 M with out = M @ in for the tile-local stage group."""
    if direction not in ("dit", "dif"):
        raise ValueError(f"unknown direction {direction!r}")
    logt = _log2_exact(tile)
    spans = [1 << s for s in range(logt)]
    if direction == "dif":
        spans.reverse()
    m = np.eye(tile, dtype=np.complex128)
    cols = []
    for t in range(tile):
        v = m[:, t].copy()
        for h in spans:
            v = _stage(v, h, direction)
        cols.append(v)
    return np.stack(cols, axis=1)


def local_matrix_planar(tile: int, direction: str = "dit"):
    """(MT_r, MT_i) float32 with out_row = in_row @ MT (row-vector form)."""
    mt = local_matrix(tile, direction).T.copy()
    return (np.ascontiguousarray(mt.real, dtype=np.float32),
            np.ascontiguousarray(mt.imag, dtype=np.float32))


def tail_groups(tile: int, logn: int, glog: int, maxp: int):
    """Partition tail stages n = tile .. N/2 into (n0, g) execution groups and
    single stages: greedily take the largest 2..glog consecutive stages whose
    period n0 << g <= maxp, else one single stage."""
    if glog < 1:
        raise ValueError(f"glog must be >= 1, got {glog}")
    stages = [1 << s for s in range(_log2_exact(tile), logn)]
    groups, singles = [], []
    i = 0
    while i < len(stages):
        n0 = stages[i]
        take = next((s for s in range(min(glog, len(stages) - i), 1, -1) if (n0 << s) <= maxp), 0)
        if take:
            groups.append((n0, take))
            i += take
        else:
            singles.append(n0)
            i += 1
    return groups, singles
