"""Runner functions of the reference API, executed by libbfft.so on B200.

Every public runner of the reference's ``src/xpu/runner.py`` exists here with
the same name, arguments, validation and result; each one resolves (and
caches) a native plan for its flow and executes it on the tensor's current
CUDA stream through the C ABI.  How each flow maps onto B200 kernels:

* ``fft_dit`` / ``fft_dif`` / ``fft_*_batch`` (M0 / M4): one radix-2 global
  stage per launch, bit reversal folded into the first DIT / last DIF stage,
  spread or folded batch grids -- the reference's stage cascade.
* ``fft_*_radix4[_batch]`` (M5): radix-4 global stages with the mixed digit
  reversal folded in, plus the radix-2 tail for odd log2 N.
* ``fft_dit_fused`` (M1): the first log2(tile) DIT stages as one CTA-resident
  pass (the bit reversal folded into its loads), then radix-2 global stages.
* ``fft_*_matrix[_batch]`` (M2, "batch local-fused core"): the local group of
  log2(tile) stages as one CTA-resident pass; the remaining stages are grouped
  into the fewest further column passes of up to 512 points each (the size the
  TMA-staged column pass covers), so N <= 4096 with tile = N is a single HBM
  round trip, N <= 2^21 with tile 4096 two, and N = 2^30 with tile 256 four.
* ``fft_*_grouped`` (M3): the local pass plus the reference's tail partition
  (``tail_groups``): each execution group is one pass, leftovers radix-2 stages.

The ``block`` argument keeps its meaning for the global-stage kernels (threads
per CTA); the CTA-resident passes size themselves from the sub-FFT length.
A ``twiddle`` argument is validated like the reference's and otherwise unused:
the library computes its tables in float64 and rounds once.
"""
from __future__ import annotations

import math
import random
import threading
import time
from collections import OrderedDict

import torch

from . import _lib
from .context import device_ready, xpu_context  # noqa: F401  (re-exported API)
from .validate import log2_exact, validate_batch_input, validate_input, validate_twiddle

DEFAULT_BLOCK = 1024

_PLANS: "OrderedDict[tuple, _lib.NativePlan]" = OrderedDict()
_PLANS_LOCK = threading.Lock()
_PLANS_MAX = 256


def native_plan(runner: str, direction: str, n: int, batch: int, device: int, **knobs) -> _lib.NativePlan:
    """Cached native plan for one runner configuration (LRU, per device)."""
    key = (runner, direction, int(n), int(batch), int(device), tuple(sorted(knobs.items())))
    with _PLANS_LOCK:
        p = _PLANS.get(key)
        if p is not None:
            _PLANS.move_to_end(key)
            return p
    desc = _lib.make_desc(runner, direction, n, batch, device=device, **knobs)
    with torch.cuda.device(device):
        p = _lib.NativePlan(desc)
    with _PLANS_LOCK:
        _PLANS[key] = p
        while len(_PLANS) > _PLANS_MAX:
            _PLANS.popitem(last=False)
    return p


def execute_native(plan: _lib.NativePlan, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Enqueue one execution of ``plan`` on x's current stream (workspace from
    torch's caching allocator, released to the same stream)."""
    dev = x.device
    ws = None
    if plan.workspace_bytes:
        ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    plan.execute(x.data_ptr(), out.data_ptr(), ws.data_ptr() if ws is not None else 0,
                 plan.workspace_bytes, stream)
    return out


def _device_index(x: torch.Tensor) -> int:
    return x.device.index if x.device.index is not None else torch.cuda.current_device()


def _c2c(runner: str, direction: str, x: torch.Tensor, batch: int, **knobs) -> torch.Tensor:
    plan = native_plan(runner, direction, x.shape[-1], batch, _device_index(x), **knobs)
    out = torch.empty_like(x)
    return execute_native(plan, x, out)


def _check_block(block) -> int:
    if not isinstance(block, int) or block <= 0 or block & (block - 1):
        raise ValueError(f"block must be a positive power of two, got {block!r}")
    return block


def twiddle_tables(n: int, device):
    """(cos, sin) float32 tables of exp(-2j pi idx / n), idx < n/2
    (reference: runner.py:93-97; here float64 angles rounded once)."""
    log2_exact(n)
    device = torch.device(device)
    half = n >> 1
    w = torch.empty(max(half, 1), dtype=torch.complex64, device=device)
    if half:
        L = _lib.load()
        _lib.check(L.bfft_twiddle_table(w.data_ptr(), n, half, _dev(device),
                                        torch.cuda.current_stream(device).cuda_stream),
                   "twiddle_table")
    w = w[:half]
    return w.real.contiguous(), w.imag.contiguous()


def _dev(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


# ----------------------------------------------------------------- rank-1 runners

def fft_dit(x: torch.Tensor, block: int = DEFAULT_BLOCK, twiddle=None) -> torch.Tensor:
    """M0: DIT radix-2 global stages, bit reversal folded into stage 0 (runner.py:118-163)."""
    validate_input(x, "x", block=block)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dit", "dit", x, 1, block=block)


def fft_dif(x: torch.Tensor, block: int = DEFAULT_BLOCK, twiddle=None) -> torch.Tensor:
    """M0: DIF radix-2 global stages, bit reversal folded into the last stage (runner.py:166-206)."""
    validate_input(x, "x", block=block)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dif", "dif", x, 1, block=block)


def fft_dit_fused(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, twiddle=None) -> torch.Tensor:
    """M1: first log2(tile) DIT stages in one CTA-resident pass, M0 tail (runner.py:209-295)."""
    validate_input(x, "x", block=block)
    if tile <= 1:
        return fft_dit(x, block=block, twiddle=twiddle)
    log2_exact(tile)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dit_fused", "dit", x, 1, block=block, tile=tile)


def _matrix_knobs(n: int, tile: int, rows: int) -> None:
    log2_exact(tile)
    if rows > 1:
        log2_exact(rows)


def fft_dit_matrix(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                   twiddle=None) -> torch.Tensor:
    """M2: local group of log2(tile) DIT stages resident on chip + grouped tail (runner.py:379-442)."""
    validate_input(x, "x", block=block)
    if tile <= 1:
        return fft_dit(x, block=block, twiddle=twiddle)
    _matrix_knobs(x.numel(), tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dit_matrix", "dit", x, 1, block=block, tile=tile, rows=max(rows, 1))


def fft_dif_matrix(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                   twiddle=None) -> torch.Tensor:
    """M2 DIF mirror: grouped tail first, then the local group + bit reversal (runner.py:445-502)."""
    validate_input(x, "x", block=block)
    if tile <= 1:
        return fft_dif(x, block=block, twiddle=twiddle)
    _matrix_knobs(x.numel(), tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dif_matrix", "dif", x, 1, block=block, tile=tile, rows=max(rows, 1))


def fft_dit_grouped(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                    glog: int = 2, maxp: int = 4096, cells: int = 1, twiddle=None) -> torch.Tensor:
    """M3: local group + tail execution groups from tail_groups (runner.py:603-682)."""
    validate_input(x, "x", block=block)
    if glog < 1:
        raise ValueError(f"glog must be >= 1, got {glog}")
    if cells < 1:
        raise ValueError(f"cells must be >= 1, got {cells}")
    if tile <= 1:
        return fft_dit(x, block=block, twiddle=twiddle)
    _matrix_knobs(x.numel(), tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dit_grouped", "dit", x, 1, block=block, tile=tile, rows=max(rows, 1),
                glog=glog, maxp=maxp, cells=cells)


def fft_dif_grouped(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                    glog: int = 2, maxp: int = 4096, cells: int = 1, twiddle=None) -> torch.Tensor:
    """M3 DIF mirror (runner.py:685-752)."""
    validate_input(x, "x", block=block)
    if glog < 1:
        raise ValueError(f"glog must be >= 1, got {glog}")
    if cells < 1:
        raise ValueError(f"cells must be >= 1, got {cells}")
    if tile <= 1:
        return fft_dif(x, block=block, twiddle=twiddle)
    _matrix_knobs(x.numel(), tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dif_grouped", "dif", x, 1, block=block, tile=tile, rows=max(rows, 1),
                glog=glog, maxp=maxp, cells=cells)


def fft_dit_radix4(x: torch.Tensor, block: int = DEFAULT_BLOCK, twiddle=None) -> torch.Tensor:
    """M5: radix-4 DIT global stages, digit reversal folded in (runner.py:1399-1469)."""
    validate_input(x, "x", block=block)
    if x.numel() < 4:
        raise ValueError(f"radix-4 requires N >= 4, got N={x.numel()}")
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dit_radix4", "dit", x, 1, block=block)


def fft_dif_radix4(x: torch.Tensor, block: int = DEFAULT_BLOCK, twiddle=None) -> torch.Tensor:
    """M5: radix-4 DIF global stages, digit reversal on the last (runner.py:1472-1540)."""
    validate_input(x, "x", block=block)
    if x.numel() < 4:
        raise ValueError(f"radix-4 requires N >= 4, got N={x.numel()}")
    if twiddle is not None:
        validate_twiddle(twiddle, x.numel(), x.device)
    return _c2c("fft_dif_radix4", "dif", x, 1, block=block)


# ----------------------------------------------------------------- batched runners

def fft_dit_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, variant: str = "spread",
                  twiddle=None) -> torch.Tensor:
    """M4: batched DIT stage cascade, spread (Ud=B) or folded (Td=B) (runner.py:781-841)."""
    b, n = validate_batch_input(x, block, variant)
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dit_batch", "dit", x, b, block=block, variant=variant)


def fft_dif_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, variant: str = "spread",
                  twiddle=None) -> torch.Tensor:
    """M4 DIF mirror (runner.py:844-896)."""
    b, n = validate_batch_input(x, block, variant)
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dif_batch", "dif", x, b, block=block, variant=variant)


def _spread_only(name: str, variant: str) -> None:
    if variant != "spread":
        raise ValueError(f"{name} lowers variant='spread' (Ud=B) only; got variant={variant!r}")


def fft_dit_matrix_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                         variant: str = "spread", twiddle=None) -> torch.Tensor:
    """M2 batch: the batch local-fused core (runner.py:956-1035)."""
    b, n = validate_batch_input(x, block, variant)
    _spread_only("fft_dit_matrix_batch", variant)
    if tile <= 1:
        return fft_dit_batch(x, block=block, variant=variant, twiddle=twiddle)
    _matrix_knobs(n, tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dit_matrix_batch", "dit", x, b, block=block, tile=tile, rows=max(rows, 1))


def fft_dif_matrix_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64, rows: int = 8,
                         variant: str = "spread", twiddle=None) -> torch.Tensor:
    """M2 batch DIF mirror (runner.py:1038-1109)."""
    b, n = validate_batch_input(x, block, variant)
    _spread_only("fft_dif_matrix_batch", variant)
    if tile <= 1:
        return fft_dif_batch(x, block=block, variant=variant, twiddle=twiddle)
    _matrix_knobs(n, tile, rows)
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dif_matrix_batch", "dif", x, b, block=block, tile=tile, rows=max(rows, 1))


def fft_dit_matrix_packet_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, tile: int = 64,
                                rows: int = 8, packets: int = 2, twiddle=None) -> torch.Tensor:
    """Experimental M2 packet loop of the reference (runner.py:1271-1364): same
    contract (packets a power of two <= 2 dividing B); on B200 every CTA already
    owns several sub-FFTs, so it executes the batch local-fused core."""
    b, n = validate_batch_input(x, block, "spread")
    if packets < 1 or packets & (packets - 1):
        raise ValueError(f"packets must be a power of two, got {packets}")
    if packets > 2:
        raise ValueError(f"packets={packets} exceeds the ceiling of 2 of this experimental flow")
    if b % packets:
        raise ValueError(f"packets={packets} must divide batch B={b}")
    return fft_dit_matrix_batch(x, block=block, tile=tile, rows=rows, twiddle=twiddle)


def fft_dit_radix4_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, variant: str = "spread",
                         twiddle=None) -> torch.Tensor:
    """M5 batch DIT (runner.py:1112-1190)."""
    b, n = validate_batch_input(x, block, variant)
    _spread_only("fft_dit_radix4_batch", variant)
    if n < 4:
        raise ValueError(f"radix-4 requires N >= 4, got N={n}")
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dit_radix4_batch", "dit", x, b, block=block)


def fft_dif_radix4_batch(x: torch.Tensor, block: int = DEFAULT_BLOCK, variant: str = "spread",
                         twiddle=None) -> torch.Tensor:
    """M5 batch DIF (runner.py:1193-1268)."""
    b, n = validate_batch_input(x, block, variant)
    _spread_only("fft_dif_radix4_batch", variant)
    if n < 4:
        raise ValueError(f"radix-4 requires N >= 4, got N={n}")
    if twiddle is not None:
        validate_twiddle(twiddle, n, x.device)
    return _c2c("fft_dif_radix4_batch", "dif", x, b, block=block)


def bit_reverse_permute(x: torch.Tensor, block: int = DEFAULT_BLOCK) -> torch.Tensor:
    """Y[i] = X[bitrev(i)] (runner.py:1542-1552); rank-2 input permutes each row."""
    if isinstance(x, torch.Tensor) and x.dim() == 2:
        b, n = validate_batch_input(x, block, "spread")
    else:
        validate_input(x, "x", block=block, require_complex=True)
        b, n = 1, x.numel()
    y = torch.empty_like(x)
    L = _lib.load()
    _lib.check(L.bfft_bit_reverse_permute(x.data_ptr(), y.data_ptr(), n, b, _device_index(x),
                                          torch.cuda.current_stream(x.device).cuda_stream),
               "bit_reverse_permute")
    return y


# ----------------------------------------------------------------- real epilogues

def _validate_real_half(x: torch.Tensor, n: int, bins: int, name: str) -> None:
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != torch.complex64:
        raise TypeError(f"{name} must be complex64, got {x.dtype}")
    if x.device.type != "cuda":
        raise ValueError(f"{name} must be on a CUDA device, got {x.device}")
    if x.dim() not in (1, 2):
        raise ValueError(f"{name} must be rank-1 or rank-2, got dim={x.dim()}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    log2_exact(n)
    if n < 4:
        raise ValueError(f"dedicated real flow needs N >= 4, got {n}")
    if x.shape[-1] != bins:
        raise ValueError(f"{name} last dim {x.shape[-1]} != expected {bins}")


def r2c_stitch(z: torch.Tensor, n: int, scale: float = 1.0, block: int = DEFAULT_BLOCK) -> torch.Tensor:
    """Half-length FFT of packed pairs -> (N/2+1) spectrum (runner.py:1687-1715)."""
    _validate_real_half(z, n, n >> 1, "z")
    _check_block(block)
    rows = 1 if z.dim() == 1 else z.shape[0]
    out = torch.empty((*z.shape[:-1], (n >> 1) + 1), dtype=torch.complex64, device=z.device)
    _lib.check(_lib.load().bfft_r2c_stitch(z.data_ptr(), out.data_ptr(), n, rows, float(scale),
                                           _device_index(z), torch.cuda.current_stream(z.device).cuda_stream),
               "r2c_stitch")
    return out


def c2r_pre(xh: torch.Tensor, n: int, block: int = DEFAULT_BLOCK) -> torch.Tensor:
    """Half spectrum -> pre-twiddled N/2-point core input (runner.py:1718-1742)."""
    _validate_real_half(xh, n, (n >> 1) + 1, "xh")
    _check_block(block)
    rows = 1 if xh.dim() == 1 else xh.shape[0]
    out = torch.empty((*xh.shape[:-1], n >> 1), dtype=torch.complex64, device=xh.device)
    _lib.check(_lib.load().bfft_c2r_pre(xh.data_ptr(), out.data_ptr(), n, rows, _device_index(xh),
                                        torch.cuda.current_stream(xh.device).cuda_stream), "c2r_pre")
    return out


def c2r_unpack(u: torch.Tensor, n: int, scale: float = 1.0, block: int = DEFAULT_BLOCK) -> torch.Tensor:
    """Half-length FFT -> N interleaved real samples (runner.py:1745-1767)."""
    _validate_real_half(u, n, n >> 1, "u")
    _check_block(block)
    rows = 1 if u.dim() == 1 else u.shape[0]
    out = torch.empty((*u.shape[:-1], n), dtype=torch.float32, device=u.device)
    _lib.check(_lib.load().bfft_c2r_unpack(u.data_ptr(), out.data_ptr(), n, rows, float(scale),
                                           _device_index(u), torch.cuda.current_stream(u.device).cuda_stream),
               "c2r_unpack")
    return out


def r2c_stitch_ref(z: torch.Tensor, n: int, scale: float = 1.0) -> torch.Tensor:
    """torch reference of r2c_stitch (runner.py:1776-1797), usable on CPU."""
    n2 = n >> 1
    if z.shape[-1] != n2:
        raise ValueError(f"z last dim {z.shape[-1]} != N/2 ({n2})")
    k = torch.arange(n2 + 1, device=z.device)
    j = (n2 - k) % n2
    ik = torch.where(k == n2, torch.zeros_like(k), k)
    zr, zi = z.real, z.imag
    ar = 0.5 * (zr[..., ik] + zr[..., j])
    ai = 0.5 * (zi[..., ik] - zi[..., j])
    cr = 0.5 * (zr[..., ik] - zr[..., j])
    ci = 0.5 * (zi[..., ik] + zi[..., j])
    ang = -2.0 * math.pi * k.double() / n
    wr, wi = torch.cos(ang).float(), torch.sin(ang).float()
    xr = ar + wr * ci + wi * cr
    xi = ai - wr * cr + wi * ci
    xi = torch.where((k == 0) | (k == n2), torch.zeros_like(xi), xi)
    return torch.complex(xr * scale, xi * scale)


def c2r_pre_ref(xh: torch.Tensor, n: int) -> torch.Tensor:
    """torch reference of c2r_pre (runner.py:1800-1821)."""
    n2 = n >> 1
    if xh.shape[-1] != n2 + 1:
        raise ValueError(f"xh last dim {xh.shape[-1]} != N/2+1 ({n2 + 1})")
    k = torch.arange(n2, device=xh.device)
    j = n2 - k
    xr, xi = xh.real, xh.imag
    xkr, xki = xr[..., k], torch.where(k == 0, torch.zeros_like(xi[..., k]), xi[..., k])
    xjr, xji = xr[..., j], torch.where(j == n2, torch.zeros_like(xi[..., j]), xi[..., j])
    ar, ai = 0.5 * (xkr + xjr), 0.5 * (xki - xji)
    cr, ci = 0.5 * (xkr - xjr), 0.5 * (xki + xji)
    ang = 2.0 * math.pi * k.double() / n
    wr, wi = torch.cos(ang).float(), torch.sin(ang).float()
    return torch.complex(ar - (wr * ci + wi * cr), ai + (wr * cr - wi * ci))


def c2r_unpack_ref(u: torch.Tensor, n: int, scale: float = 1.0) -> torch.Tensor:
    """torch reference of c2r_unpack (runner.py:1824-1834)."""
    n2 = n >> 1
    if u.shape[-1] != n2:
        raise ValueError(f"u last dim {u.shape[-1]} != N/2 ({n2})")
    k = torch.arange(n2, device=u.device)
    m = torch.where(k == 0, torch.zeros_like(k), n2 - k)
    out = torch.empty((*u.shape[:-1], n), dtype=torch.float32, device=u.device)
    out[..., 0::2] = u.real[..., m] * scale
    out[..., 1::2] = u.imag[..., m] * scale
    return out


# ----------------------------------------------------------------- device / timing

def device_name() -> str:
    if not device_ready():
        return "cpu"
    p = torch.cuda.get_device_properties(torch.cuda.current_device())
    return f"{p.name} (sm_{p.major}{p.minor}, {p.multi_processor_count} SMs, {p.total_memory >> 30} GiB)"


def _sync():
    if device_ready():
        torch.cuda.synchronize()


def time_call(fn, warmup: int = 5, iters: int = 20) -> float:
    """Median API wall time in ms (dispatch + launches + synchronisation)."""
    for _ in range(warmup):
        fn()
    _sync()
    samples = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        _sync()
        samples.append((time.perf_counter() - t0) * 1e3)
    samples.sort()
    return samples[len(samples) // 2]


def time_call_detailed(fn, warmup: int = 10, trials: int = 50, seed: int = 0) -> dict:
    """Interleaved trials: API wall time and CUDA-event device time, reported
    separately (reference: runner.py:1576-1635)."""
    for _ in range(warmup):
        fn()
    _sync()
    api, kern = [], []
    order = list(range(trials))
    random.Random(seed).shuffle(order)
    for _ in order:
        if device_ready():
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            api.append((time.perf_counter() - t0) * 1e3)
            kt = s.elapsed_time(e)
            if kt > 0:
                kern.append(kt)
        else:
            t0 = time.perf_counter()
            fn()
            api.append((time.perf_counter() - t0) * 1e3)

    def stats(xs):
        if not xs:
            return None
        xs = sorted(xs)
        return {"median": xs[len(xs) // 2], "min": xs[0], "p10": xs[max(0, int(0.1 * len(xs)))],
                "p90": xs[min(len(xs) - 1, int(0.9 * len(xs)))], "trials": len(xs)}

    return {"api_ms": stats(api), "kernel_ms": stats(kern),
            "metric_note": "api_ms = synchronized wall time; kernel_ms = CUDA event device time",
            "raw": {"api_ms": api, "kernel_ms": kern}}
