"""CPU restatement of the distributed 4-step phases -- TEST INFRASTRUCTURE ONLY.

The checker for ``bfft_dist_phase`` (``kunlunxin-fft_b200/csrc/bfft_dist.cu``)
and the stand-in device work of the host orchestration tests
(``bfft.dist.DistributedFFT`` run over ``gloo`` on CPU).  Only ``tests/`` may
import it; the product path never does.

The decomposition is the reference's hybrid 4-step (N = N1 * N2,
``src/xpu/adapter_hybrid.py:224-270``: stride gather, length-N1 sub-FFTs,
twiddle W_N^{n2 k1} built in float64, length-N2 sub-FFTs, transpose to
natural order ``X[k2 N1 + k1]``), here spread over P ranks holding
contiguous slabs, with the three transposes that cross ranks done as
all-to-alls between the phases.  Each phase below is written directly from
that index algebra in numpy (row FFTs in float64 via ``numpy.fft``).
"""
from __future__ import annotations

import numpy as np


def norm_scale(n: int, transform_direction: str, norm: str) -> float:
    """torch.fft norm convention (src/xpu/entry.py:81-102)."""
    if norm == "ortho":
        return 1.0 / np.sqrt(n)
    if (norm == "forward" and transform_direction == "forward") or \
            (norm == "backward" and transform_direction == "inverse"):
        return 1.0 / n
    return 1.0


class NumpyPhases:
    """Phases 0..3 of one rank on host arrays (any complex dtype).

    ``phase(k, x)`` takes the rank's input of phase k (a 1-D array of N/P
    values: the local slab for phase 0, the receive buffer of the previous
    all-to-all otherwise) and returns its output (the send buffer of the next
    all-to-all, or the local output slab after phase 3)."""

    def __init__(self, n1: int, n2: int, nranks: int, rank: int, transform_direction: str = "forward",
                 norm: str = "backward", dtype=np.complex128):
        if n1 % nranks or n2 % nranks:
            raise ValueError("nranks must divide n1 and n2")
        self.n1, self.n2, self.p, self.r = n1, n2, nranks, rank
        self.m1, self.m2 = n1 // nranks, n2 // nranks
        self.n = n1 * n2
        self.inv = transform_direction == "inverse"
        self.scale = norm_scale(self.n, transform_direction, norm)
        self.dtype = dtype

    def _fft_rows(self, a: np.ndarray) -> np.ndarray:
        return np.fft.fft(a.astype(np.complex128), axis=-1).astype(self.dtype)

    def phase(self, k: int, x: np.ndarray) -> np.ndarray:
        p, m1, m2, n1, n2 = self.p, self.m1, self.m2, self.n1, self.n2
        x = np.asarray(x)
        if k == 0:  # x_r[i][n2] -> [n2][i]
            a = x.reshape(m1, n2)
            if self.inv:
                a = np.conj(a)
            return np.ascontiguousarray(a.T).reshape(-1).astype(self.dtype)
        if k == 1:  # recv[p][n2'][i] -> [n2'][n1] -> FFT -> [k1][n2'] * W_N^{n2 k1}
            rows = x.reshape(p, m2, m1).transpose(1, 0, 2).reshape(m2, n1)
            v = self._fft_rows(rows)
            n2g = (self.r * m2 + np.arange(m2, dtype=np.int64))[:, None]
            k1 = np.arange(n1, dtype=np.int64)[None, :]
            e = (n2g * k1) % self.n
            tw = np.exp(-2j * np.pi * e.astype(np.float64) / self.n).astype(self.dtype)
            return np.ascontiguousarray((v * tw).T).reshape(-1).astype(self.dtype)
        if k == 2:  # recv[s][k1'][n2'] -> [k1'][n2] -> FFT -> [k2][k1']
            rows = x.reshape(p, m1, m2).transpose(1, 0, 2).reshape(m1, n2)
            h = self._fft_rows(rows)
            return np.ascontiguousarray(h.T).reshape(-1).astype(self.dtype)
        if k == 3:  # recv[s][k2'][k1'] -> [k2'][k1]
            out = x.reshape(p, m2, m1).transpose(1, 0, 2).reshape(-1)
            if self.inv:
                out = np.conj(out)
            return (out * self.scale).astype(self.dtype)
        if k == 4:  # transposed output: recv[s][k1'][n2'] -> [k1'][n2] -> FFT -> [k1'][k2]
            rows = x.reshape(p, m1, m2).transpose(1, 0, 2).reshape(m1, n2)
            h = self._fft_rows(rows).reshape(-1)
            if self.inv:
                h = np.conj(h)
            return (h * self.scale).astype(self.dtype)
        raise ValueError(f"phase must be 0..4, got {k}")


def transposed_slab(X: np.ndarray, n1: int, n2: int, nranks: int, rank: int) -> np.ndarray:
    """What rank ``rank`` holds after the transposed-output flow, given the
    whole transform X in natural order: the (N1/P) x N2 block
    out[k1'][k2] = X[k2 N1 + rank N1/P + k1']."""
    m1 = n1 // nranks
    return np.ascontiguousarray(X.reshape(n2, n1).T[rank * m1:(rank + 1) * m1, :]).reshape(-1)


def emulate(x: np.ndarray, n1: int, n2: int, nranks: int, transform_direction: str = "forward",
            norm: str = "backward", phase_fns=None, output_order: str = "natural") -> np.ndarray:
    """Run all ranks' phases in one process with the all-to-alls done by
    array slicing; returns the concatenated output slabs (natural order: the
    whole transform; transposed: the ranks' ``transposed_slab`` blocks one
    after another).  ``phase_fns[r](k, x)`` defaults to ``NumpyPhases``."""
    n = n1 * n2
    slab = n // nranks
    chunk = slab // nranks
    if phase_fns is None:
        phase_fns = [NumpyPhases(n1, n2, nranks, r, transform_direction, norm).phase for r in range(nranks)]
    bufs = [x[r * slab:(r + 1) * slab] for r in range(nranks)]
    seq = (0, 1, 2, 3) if output_order == "natural" else (0, 1, 4)
    for k in seq:
        outs = [phase_fns[r](k, bufs[r]) for r in range(nranks)]
        if k in (3, 4):
            return np.concatenate([np.asarray(o) for o in outs])
        bufs = [np.concatenate([np.asarray(outs[s])[r * chunk:(r + 1) * chunk] for s in range(nranks)])
                for r in range(nranks)]
    raise AssertionError("unreachable")
