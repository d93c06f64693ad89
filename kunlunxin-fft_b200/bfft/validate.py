"""Input validation for the public FFT API (reference: src/xpu/validate.py).

Bad inputs are rejected before any launch with the reference's exception
types: TypeError for a non-tensor or a wrong dtype, ValueError for rank,
contiguity, device or a non-power-of-two length, RuntimeError when the CUDA
device stack is unavailable.
"""
from __future__ import annotations

import torch

from .context import device_ready


def log2_exact(n: int) -> int:
    if n <= 0 or (n & (n - 1)) != 0:
        raise ValueError(f"size must be a positive power of two, got {n}")
    return int(n.bit_length() - 1)


def validate_input(x, name: str = "x", *, allow_n: int | None = None, block: int | None = None,
                   require_complex: bool = True) -> None:
    """Rank-1, complex64, contiguous, on a CUDA device, power-of-two length."""
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(x).__name__}")
    if x.dim() != 1:
        raise ValueError(f"{name} must be 1-D, got {x.dim()}-D (shape {tuple(x.shape)}); "
                         "use the batched runners for (B, N) inputs")
    if require_complex and x.dtype != torch.complex64:
        raise TypeError(f"{name} must be complex64, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous; got a non-contiguous view. "
                         "Clone or contiguous() it before calling")
    if not device_ready():
        raise RuntimeError("CUDA device stack not available; cannot validate device")
    if x.device.type != "cuda":
        raise ValueError(f"{name} must be on a CUDA device, got device={x.device}")
    n = x.numel()
    log2_exact(n)
    if allow_n is not None and n != allow_n:
        raise ValueError(f"{name} length {n} != expected {allow_n}")
    if block is not None:
        log2_exact(block)


def validate_batch_input(x, block: int, variant: str):
    """Batched runner contract: contiguous (B, N) complex64 on CUDA, power-of-two
    axes (reference: src/xpu/runner.py:757-778)."""
    if variant not in ("spread", "folded"):
        raise ValueError(f"variant must be 'spread' or 'folded', got {variant!r}")
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != torch.complex64:
        raise TypeError(f"x must be complex64, got {x.dtype}")
    if not device_ready():
        raise RuntimeError("CUDA device stack not available")
    if x.device.type != "cuda":
        raise ValueError(f"x must be on a CUDA device, got {x.device}")
    if x.dim() != 2:
        raise ValueError(f"x must be rank-2 (batch, length), got dim={x.dim()}")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    if block <= 0 or (block & (block - 1)) != 0:
        raise ValueError(f"block must be a power of two, got {block}")
    b, n = x.shape
    if b < 1:
        raise ValueError(f"batch must be >= 1, got {b}")
    log2_exact(b)
    log2_exact(n)
    return int(b), int(n)


def validate_twiddle(tw, n: int, device) -> None:
    """A (cos, sin) pair from twiddle_tables(n): float32, N/2 entries, same device."""
    if not isinstance(tw, tuple) or len(tw) != 2:
        raise TypeError("twiddle must be a (cos, sin) tuple from twiddle_tables()")
    for t, nm in zip(tw, ("cos", "sin")):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"twiddle {nm} must be a torch.Tensor")
        if t.dtype != torch.float32:
            raise TypeError(f"twiddle {nm} must be float32, got {t.dtype}")
        if t.device != device:
            raise ValueError(f"twiddle {nm} device {t.device} != input device {device}")
        if t.numel() != n >> 1:
            raise ValueError(f"twiddle {nm} length {t.numel()} != N/2 ({n >> 1})")
