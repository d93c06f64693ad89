"""CPU oracle for the B200 FFT library -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import
it.  The product path (``bfft``) never imports anything under ``oracle/`` and
fails loudly when its CUDA library is missing.

Two layers:

* ``liboracle.so`` (``fft_oracle.c``): a C restatement of the reference's FP32
  arithmetic -- radix-2 / radix-4 stage cascades, the bit and digit reversal
  index maps, and the real-transform epilogues -- plus a float64 radix-2 FFT
  restating ``include/butterfly/fft.hpp``.
* this file: the reference's host-side composition restated in numpy --
  ``norm_scale`` and the inverse conjugate trick (``src/xpu/entry.py``), the
  dedicated and compat real flows, the M2 local matrix
  (``src/xpu/matrices.py``) and the hybrid 4-step decomposition
  (``src/xpu/adapter_hybrid.py``).

Pinning: ``tests/test_oracle.py`` checks every function here against golden
vectors produced by running the reference itself (``tests/golden/``) and
against the reference's own C++ FFT compiled in place
(``oracle/_ref/libbutterfly_ref.so``).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libbutterfly_ref.so")

_lib = None
_ref = None


def _build(target: str) -> None:
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)


def lib() -> ctypes.CDLL:
    """The compiled C restatement (built on first use when gcc is present)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            _build("oracle")
        L = ctypes.CDLL(LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        f64p = ctypes.POINTER(ctypes.c_double)
        i64 = ctypes.c_int64
        for name in ("bfo_bit_reverse", "bfo_dit_digit_reverse", "bfo_dif_digit_reverse"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.c_uint32, ctypes.c_int]
            fn.restype = ctypes.c_uint32
        L.bfo_index_table.argtypes = [ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_uint32)]
        L.bfo_twiddle_f32.argtypes = [i64, i64, f32p, f32p]
        for name in ("bfo_fft_radix2_f32", "bfo_fft_radix4_f32"):
            fn = getattr(L, name)
            fn.argtypes = [f32p, f32p, i64, i64, ctypes.c_int]
            fn.restype = ctypes.c_int
        L.bfo_bitrev_permute.argtypes = [f32p, f32p, i64, i64]
        L.bfo_r2c_stitch_f32.argtypes = [f32p, f32p, i64, i64, ctypes.c_float]
        L.bfo_c2r_pre_f32.argtypes = [f32p, f32p, i64, i64]
        L.bfo_c2r_unpack_f32.argtypes = [f32p, f32p, i64, i64, ctypes.c_float]
        L.bfo_fft_f64.argtypes = [f64p, f64p, i64, i64, ctypes.c_int, ctypes.c_int]
        L.bfo_fft_f64.restype = ctypes.c_int
        _lib = L
    return _lib


def reference_lib() -> ctypes.CDLL | None:
    """The reference's own C++ CPU FFT, compiled in place (None if not built)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB_PATH):
            return None
        L = ctypes.CDLL(REF_LIB_PATH)
        L.ref_bit_reverse.argtypes = [ctypes.c_uint32, ctypes.c_int]
        L.ref_bit_reverse.restype = ctypes.c_uint32
        f64p = ctypes.POINTER(ctypes.c_double)
        L.ref_fft_c128.argtypes = [f64p, f64p, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int, ctypes.c_int]
        L.ref_fft_c128.restype = ctypes.c_int
        _ref = L
    return _ref


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _dp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _rows(x):
    """(B, N) contiguous view of a rank-1 or rank-2 array."""
    x = np.ascontiguousarray(x)
    return x.reshape(1, -1) if x.ndim == 1 else x


# ------------------------------------------------------------------ index maps

def index_table(kind: str, bits: int) -> np.ndarray:
    """bitrev / dit_digrev / dif_digrev permutation table of 2**bits entries."""
    k = {"bitrev": 0, "dit_digrev": 1, "dif_digrev": 2}[kind]
    out = np.empty(1 << bits, np.uint32)
    lib().bfo_index_table(k, bits, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return out


def twiddle_f32(n: int, count: int | None = None):
    count = n // 2 if count is None else count
    wr = np.empty(count, np.float32)
    wi = np.empty(count, np.float32)
    lib().bfo_twiddle_f32(n, count, _fp(wr), _fp(wi))
    return wr, wi


# ------------------------------------------------------------------ cascades

def fft_radix2_f32(x: np.ndarray, dif: bool = False) -> np.ndarray:
    """M0/M4 radix-2 FP32 cascade (src/xpu/runner.py:118-206, :781-896)."""
    r = _rows(x.astype(np.complex64))
    y = np.empty_like(r)
    rc = lib().bfo_fft_radix2_f32(_fp(r.view(np.float32)), _fp(y.view(np.float32)),
                                  r.shape[1], r.shape[0], int(dif))
    if rc:
        raise ValueError("length must be a power of two")
    return y.reshape(x.shape)


def fft_radix4_f32(x: np.ndarray, dif: bool = False) -> np.ndarray:
    """M5 radix-4 FP32 cascade (src/xpu/runner.py:1112-1268, :1367-1540)."""
    r = _rows(x.astype(np.complex64))
    y = np.empty_like(r)
    rc = lib().bfo_fft_radix4_f32(_fp(r.view(np.float32)), _fp(y.view(np.float32)),
                                  r.shape[1], r.shape[0], int(dif))
    if rc:
        raise ValueError("radix-4 needs a power-of-two length >= 4")
    return y.reshape(x.shape)


def fft_f64(x: np.ndarray, dif: bool = False, inverse: bool = False) -> np.ndarray:
    """Float64 radix-2 FFT restating include/butterfly/fft.hpp:28-97
    (inverse = unnormalised, +i exponent)."""
    r = _rows(x.astype(np.complex128))
    y = np.empty_like(r)
    rc = lib().bfo_fft_f64(_dp(r.view(np.float64)), _dp(y.view(np.float64)),
                           r.shape[1], r.shape[0], int(dif), 1 if inverse else -1)
    if rc:
        raise ValueError("length must be a power of two")
    return y.reshape(x.shape)


def bitrev_permute(x: np.ndarray) -> np.ndarray:
    """Y[i] = X[bitrev(i)] per row (src/xpu/kernels.py:81-97, :536-561)."""
    r = _rows(x.astype(np.complex64))
    y = np.empty_like(r)
    lib().bfo_bitrev_permute(_fp(r.view(np.float32)), _fp(y.view(np.float32)),
                             r.shape[1], r.shape[0])
    return y.reshape(x.shape)


# ------------------------------------------------------------------ real epilogues

def r2c_stitch(z: np.ndarray, n: int, scale: float = 1.0) -> np.ndarray:
    """src/xpu/kernels.py:1127-1177."""
    r = _rows(z.astype(np.complex64))
    y = np.empty((r.shape[0], n // 2 + 1), np.complex64)
    lib().bfo_r2c_stitch_f32(_fp(r.view(np.float32)), _fp(y.view(np.float32)),
                             n, r.shape[0], float(scale))
    return y if z.ndim == 2 else y[0]


def c2r_pre(xh: np.ndarray, n: int) -> np.ndarray:
    """src/xpu/kernels.py:1180-1229."""
    r = _rows(xh.astype(np.complex64))
    y = np.empty((r.shape[0], n // 2), np.complex64)
    lib().bfo_c2r_pre_f32(_fp(r.view(np.float32)), _fp(y.view(np.float32)),
                          n, r.shape[0])
    return y if xh.ndim == 2 else y[0]


def c2r_unpack(u: np.ndarray, n: int, scale: float = 1.0) -> np.ndarray:
    """src/xpu/kernels.py:1232-1258."""
    r = _rows(u.astype(np.complex64))
    y = np.empty((r.shape[0], n), np.float32)
    lib().bfo_c2r_unpack_f32(_fp(r.view(np.float32)), _fp(y), n, r.shape[0],
                             float(scale))
    return y if u.ndim == 2 else y[0]


# ------------------------------------------------------------------ host composition

def norm_scale(n: int, transform_direction: str, norm: str) -> float:
    """torch.fft norm table (src/xpu/entry.py:81-102)."""
    if norm == "ortho":
        return 1.0 / math.sqrt(n)
    if (norm, transform_direction) in (("forward", "forward"), ("backward", "inverse")):
        return 1.0 / n
    return 1.0


def local_matrix(tile: int, direction: str = "dit") -> np.ndarray:
    """Complex128 M with out = M @ in for the first log2(tile) DIT stages (on the
    bit-reversed tile) or the last log2(tile) DIF stages (src/xpu/matrices.py:64-92).
    Built column by column by pushing unit vectors through the radix-2 stages."""
    logt = int(tile).bit_length() - 1
    m = np.empty((tile, tile), np.complex128)
    for t in range(tile):
        v = np.zeros(tile, np.complex128)
        v[t] = 1.0
        stages = range(logt) if direction == "dit" else range(logt - 1, -1, -1)
        for s in stages:
            half = 1 << s
            w = np.exp(-2j * np.pi * np.arange(half) / (2 * half))
            blk = v.reshape(-1, 2 * half)
            lo, hi = blk[:, :half].copy(), blk[:, half:].copy()
            if direction == "dit":
                hi = hi * w
                v = np.concatenate((lo + hi, lo - hi), axis=1).reshape(tile)
            else:
                v = np.concatenate((lo + hi, (lo - hi) * w), axis=1).reshape(tile)
        m[:, t] = v
    return m


def hybrid_4step(x: np.ndarray, tile: int, core=None) -> np.ndarray:
    """DIT 4-step N = T*R decomposition of src/xpu/adapter_hybrid.py:224-270:
    gather (tile, t2) view, length-t2 row FFTs, twiddle w_N^{k_t*m0} (built in
    float64, cast to complex64), length-tile row FFTs, transpose to natural
    order X[k_r*T + k_t].  ``core`` is the row-FFT (defaults to the FP32
    radix-2 cascade)."""
    core = core or (lambda a: fft_radix2_f32(a))
    r = _rows(x.astype(np.complex64))
    b, n = r.shape
    t2 = n // tile
    blocks = r.reshape(b, t2, tile).transpose(0, 2, 1).reshape(b * tile, t2)
    s1 = core(np.ascontiguousarray(blocks))
    kt = np.arange(t2, dtype=np.float64)
    m0 = np.arange(tile, dtype=np.float64)
    tw = np.exp(-2j * np.pi * np.outer(kt, m0) / n).astype(np.complex64)
    grid = (s1.reshape(b, tile, t2).transpose(0, 2, 1) * tw).astype(np.complex64)
    s2 = core(np.ascontiguousarray(grid.reshape(b * t2, tile)))
    out = s2.reshape(b, t2, tile).transpose(0, 2, 1).reshape(b, n)
    return out if x.ndim == 2 else out[0]


_RADIX4 = {"fft_dit_radix4", "fft_dif_radix4", "fft_dit_radix4_batch",
           "fft_dif_radix4_batch"}


def core_fft(runner: str, z: np.ndarray, params: dict | None = None) -> np.ndarray:
    """Oracle for one runner's unnormalised forward transform.

    M0/M4 use the radix-2 cascade of their own orientation, M5 the radix-4
    cascade; M1/M2/M3 compute the same radix-2 DIT/DIF linear map (their
    grouping changes only FP32 rounding) and are checked against the radix-2
    cascade; run_hybrid uses the 4-step restatement."""
    params = params or {}
    dif = "_dif" in runner
    if runner in _RADIX4:
        return fft_radix4_f32(z, dif=dif)
    if runner == "run_hybrid":
        return hybrid_4step(z, int(params.get("tile", 64)))
    return fft_radix2_f32(z, dif=dif)


def execute(runner: str, x: np.ndarray, transform_type: str = "c2c",
            transform_direction: str = "forward", norm: str = "backward",
            real_flow: str | None = None, params: dict | None = None) -> np.ndarray:
    """Oracle of execute_fft_plan (src/xpu/entry.py:501-628) for one plan."""
    n = x.shape[-1]
    if transform_type == "c2c":
        z = np.conj(x) if transform_direction == "inverse" else x
        y = core_fft(runner, z.astype(np.complex64), params)
        s = np.float32(norm_scale(n, transform_direction, norm))
        if transform_direction == "inverse":
            return (np.conj(y) * s).astype(np.complex64)
        return (y * s).astype(np.complex64) if s != 1 else y
    if transform_type == "r2c":
        if real_flow:
            z = np.ascontiguousarray(x.astype(np.float32)).view(np.complex64)
            u = core_fft(runner, z, params)
            return r2c_stitch(u, n, norm_scale(n, "forward", norm))
        y = core_fft(runner, x.astype(np.complex64), params)
        s = np.float32(norm_scale(n, "forward", norm))
        y = (y * s).astype(np.complex64) if s != 1 else y
        return np.ascontiguousarray(y[..., : n // 2 + 1])
    if transform_type == "c2r":
        nfull = 2 * (x.shape[-1] - 1)
        if real_flow:
            zpre = c2r_pre(x, nfull)
            u = core_fft(runner, zpre, params)
            return c2r_unpack(u, nfull, 2.0 * norm_scale(nfull, "inverse", norm))
        full = hermitian_reconstruct(x, nfull)
        y = core_fft(runner, np.conj(full), params)
        s = np.float32(norm_scale(nfull, "inverse", norm))
        return np.ascontiguousarray((np.conj(y) * s).real.astype(np.float32))
    raise ValueError(transform_type)


def hermitian_reconstruct(x: np.ndarray, n: int) -> np.ndarray:
    """Full spectrum from a half spectrum, DC/Nyquist imaginary dropped
    (src/xpu/entry.py:671-696)."""
    m = n // 2 + 1
    full = np.empty(x.shape[:-1] + (n,), np.complex64)
    full[..., :m] = x
    full[..., m:] = np.conj(x[..., 1:m - 1][..., ::-1])
    full[..., 0] = full[..., 0].real
    full[..., m - 1] = full[..., m - 1].real
    return full


# ------------------------------------------------------------------ checks

def rel_l2(got, ref) -> float:
    """Relative L2 error ||got-ref|| / ||ref|| in float64 (inf if non-finite)."""
    g = np.asarray(got).astype(np.complex128)
    r = np.asarray(ref).astype(np.complex128)
    if not (np.isfinite(g).all() and np.isfinite(r).all()):
        return float("inf")
    den = np.linalg.norm(r)
    return float(np.linalg.norm(g - r) / max(den, 1e-300))


def rel_l2_rows(got, ref) -> float:
    """Worst per-transform relative L2 error over the rows of (B, N) arrays."""
    g = _rows(np.asarray(got).astype(np.complex128))
    r = _rows(np.asarray(ref).astype(np.complex128))
    if not (np.isfinite(g).all() and np.isfinite(r).all()):
        return float("inf")
    num = np.linalg.norm(g - r, axis=1)
    den = np.maximum(np.linalg.norm(r, axis=1), 1e-300)
    return float((num / den).max())


def reference_fft_c128(x: np.ndarray, dif: bool = False, threads: int = 1) -> np.ndarray:
    """Run the reference's own C++ FFT (butterfly::fft_dit / fft_dif)."""
    L = reference_lib()
    if L is None:
        raise RuntimeError("oracle/_ref/libbutterfly_ref.so not built")
    r = _rows(x.astype(np.complex128))
    y = np.empty_like(r)
    rc = L.ref_fft_c128(_dp(r.view(np.float64)), _dp(y.view(np.float64)),
                        r.shape[1], r.shape[0], int(dif), int(threads))
    if rc:
        raise ValueError("length must be a power of two")
    return y.reshape(x.shape)
