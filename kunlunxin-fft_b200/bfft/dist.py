"""Multi-GPU paths: batch sharding and the distributed 4-step transform.

The reference runs on one device; these are its single-device transforms
carried across the ranks of a ``torch.distributed`` process group, one
process per GPU (NCCL over NVLink on B200, ``gloo`` for the CPU tests).

* Batch sharding (a batched C2C / R2C / C2R job whose rows are independent):
  ``batch_shard`` gives each rank a contiguous block of rows
  (``bfft_dist_batch_shard``) and the rank runs an ordinary plan on them.  No
  collective touches the data path.
* ``DistributedFFT``: one 1-D C2C transform of N = N1 * N2 points held as
  contiguous slabs, computed with the reference's hybrid 4-step
  decomposition (``src/xpu/adapter_hybrid.py:224-270``) whose three
  transposes become all-to-alls (``all_to_all_single``, equal chunks) between
  the four device phases of ``bfft_dist_phase``.  With
  ``output_order="transposed"`` the last exchange and the two local passes
  around it are skipped: rank r ends with the (N1/P) x N2 block
  ``out[k1'][k2] = X[k2 N1 + r N1/P + k1']`` (whole columns of the N1 x N2
  output view) instead of the slab ``X[r N/P : (r+1) N/P]``.

The device phases come from libbfft.so; there is no CPU fallback.  The
``phases`` argument of ``DistributedFFT`` exists so the orchestration can be
exercised on CPU ranks with a host restatement of the phases standing in for
the device (tests only).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _lib


def _group_info(group) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def batch_shard(batch: int, world: int | None = None, rank: int | None = None, group=None) -> tuple[int, int]:
    """(first row, row count) of this rank's block of a ``batch``-row job.

    Rows are split contiguously; the first ``batch % world`` ranks take one
    extra row (the rule of ``bfft_dist_batch_shard``)."""
    if world is None or rank is None:
        w, r = _group_info(group)
        world = w if world is None else world
        rank = r if rank is None else rank
    return _lib.batch_shard(batch, world, rank)


def default_factors(n: int, world: int = 1) -> tuple[int, int]:
    """N = N1 * N2 with N1 = 2^ceil(log2 N / 2), N2 = N / N1 (2^15 x 2^15 at
    N = 2^30)."""
    if n < 4 or n & (n - 1):
        raise ValueError(f"n must be a power of two >= 4, got {n}")
    l = int(math.log2(n))
    n1 = 1 << ((l + 1) // 2)
    return n1, n // n1


class _NativePhases:
    """Device phases of one rank (bfft_dist_phase on the current stream)."""

    def __init__(self, n1: int, n2: int, world: int, rank: int, transform_direction: str, norm: str,
                 device: torch.device, row_tiles: tuple[int, int]):
        if device.type != "cuda":
            raise RuntimeError("DistributedFFT needs a CUDA device (there is no CPU fallback)")
        self.device = device
        self.plan = _lib.NativeDistPlan(n1, n2, world, rank, transform_direction=transform_direction, norm=norm,
                                        row_tiles=row_tiles, device=device.index or 0)
        self.ws = torch.empty(max(self.plan.workspace_bytes, 16), dtype=torch.uint8, device=device)
        self.natural_launches = sum(self.plan.launches[:4])
        L = self.plan.launches
        self.transposed_launches = L[0] + L[1] + L[4]
        self.launches = self.natural_launches

    def empty(self, count: int) -> torch.Tensor:
        return torch.empty(count, dtype=torch.complex64, device=self.device)

    def phase(self, k: int, x: torch.Tensor, out: torch.Tensor) -> None:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.plan.phase(k, x.data_ptr(), out.data_ptr(), self.ws.data_ptr(), self.ws.numel(), stream)


class _NativeP2PPhases(_NativePhases):
    """Device phases with every exchange fused into the transpose before it:
    results are stored over NVLink straight into the destination ranks'
    exchange buffers (CUDA IPC mappings, plain peer stores, no multicast)."""

    p2p = True

    def __init__(self, n1, n2, world, rank, transform_direction, norm, device, row_tiles, group):
        super().__init__(n1, n2, world, rank, transform_direction, norm, device, row_tiles)
        base, handle = self.plan.p2p_prepare()
        if world > 1:
            mine = torch.tensor(list(handle), dtype=torch.uint8, device=device)
            every = torch.empty(world * len(handle), dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            self.plan.p2p_attach(bytes(every.cpu().tolist()))
        else:
            self.plan.p2p_attach_pointers([base])
        # no chunk permutes (the scatters place every chunk), and phase 3 is a copy
        L, permutes = self.plan.launches, (1 if world > 1 else 0)
        self.natural_launches = L[0] + (L[1] - permutes) + (L[2] - permutes)
        self.transposed_launches = L[0] + (L[1] - permutes) + (L[4] - permutes)
        self.launches = self.natural_launches

    def phase(self, k: int, x, out) -> None:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.plan.p2p_phase(k, x.data_ptr() if x is not None else 0, out.data_ptr() if out is not None else 0,
                            self.ws.data_ptr(), self.ws.numel(), stream)


class DistributedFFT:
    """One C2C transform of ``n`` points over the ranks of ``group``.

    Rank r passes its slab ``x[r n/P : (r+1) n/P]`` (complex64, 1-D,
    contiguous, on its device) and receives ``X[r n/P : (r+1) n/P]`` of the
    transform in natural order, with the reference's ``transform_direction``
    and ``norm`` semantics (src/xpu/entry.py:81-102, :619-621).  P must be a
    power of two dividing both factors of ``n = n1 * n2``.

    ``output_order="transposed"`` (two exchanges instead of three): rank r
    receives the (N1/P) x N2 block ``out[k1'][k2] = X[k2 N1 + r N1/P + k1']``
    (``output_view`` reshapes it), for callers that consume the spectrum
    column-wise or transform back with the matching input order."""

    def __init__(self, n: int, *, n1: int | None = None, group=None, transform_direction: str = "forward",
                 norm: str = "backward", device=None, row_tiles: tuple[int, int] = (0, 0), phases=None,
                 exchange: str | None = None, output_order: str = "natural"):
        if output_order not in ("natural", "transposed"):
            raise ValueError(f"output_order must be 'natural' or 'transposed', got {output_order!r}")
        if transform_direction not in ("forward", "inverse"):
            raise ValueError(f"transform_direction must be 'forward' or 'inverse', got {transform_direction!r}")
        if norm not in ("none", "forward", "backward", "ortho"):
            raise ValueError(f"norm must be none/forward/backward/ortho, got {norm!r}")
        self.world, self.rank = _group_info(group)
        if n1 is None:
            n1, n2 = default_factors(n, self.world)
        else:
            if n1 < 2 or n1 & (n1 - 1) or n % n1:
                raise ValueError(f"n1={n1} must be a power of two dividing n={n}")
            n2 = n // n1
        if n2 < 2 or n1 % self.world or n2 % self.world:
            raise ValueError(f"world size {self.world} must divide both factors {n1} x {n2}")
        self.n, self.n1, self.n2, self.group = n, n1, n2, group
        self.slab = n // self.world
        self.transform_direction, self.norm = transform_direction, norm
        if exchange is None:
            exchange = "p2p" if self.world > 1 else "nccl"
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', got {exchange!r}")
        if phases is None:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            if exchange == "p2p":
                phases = _NativeP2PPhases(n1, n2, self.world, self.rank, transform_direction, norm, dev, row_tiles,
                                          group)
            else:
                phases = _NativePhases(n1, n2, self.world, self.rank, transform_direction, norm, dev, row_tiles)
        self.exchange = "p2p" if getattr(phases, "p2p", False) else "nccl"
        self.output_order = output_order
        self.phases = phases
        self._bufs = None
        self._flag = None

    @property
    def launches(self) -> int:
        """Device kernels one execute() enqueues on this rank."""
        key = "transposed_launches" if self.output_order == "transposed" else "natural_launches"
        return getattr(self.phases, key, getattr(self.phases, "launches", 0))

    def output_view(self, out: torch.Tensor) -> torch.Tensor:
        """``out`` as the rank's 2-D output block: (N2/P, N1) rows of
        ``X[k2 N1 + k1]`` (natural) or (N1/P, N2) with element [k1'][k2] =
        ``X[k2 N1 + r N1/P + k1']`` (transposed)."""
        if self.output_order == "transposed":
            return out.view(self.n1 // self.world, self.n2)
        return out.view(self.n2 // self.world, self.n1)

    def _buffers(self):
        if self._bufs is None:
            self._bufs = (self.phases.empty(self.slab), self.phases.empty(self.slab))
        return self._bufs

    def _barrier(self) -> None:
        """Stream-ordered: work after it starts once every rank's work before it
        has completed (an all-reduce of one word)."""
        if self.world == 1:
            return
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=self.phases.device)
        dist.all_reduce(self._flag, group=self.group)

    def _exchange(self, send: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return send
        dist.all_to_all_single(recv, send, group=self.group)
        return recv

    def execute(self, x: torch.Tensor, out: torch.Tensor | None = None, trace: list | None = None) -> torch.Tensor:
        """Enqueue one transform on the current stream.  ``trace`` (optional
        list) receives ``(step, cuda.Event)`` pairs recorded after every phase
        and exchange, for per-step device times."""
        if not isinstance(x, torch.Tensor):
            raise TypeError("x must be a torch.Tensor")
        if x.dtype != torch.complex64:
            raise TypeError(f"x must be complex64, got {x.dtype}")
        if x.dim() != 1 or x.numel() != self.slab or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous 1-D slab of {self.slab} points, got {tuple(x.shape)}")
        if out is None:
            out = self.phases.empty(self.slab)
        mids = (1, 2) if self.output_order == "natural" else (1,)
        last = 3 if self.output_order == "natural" else 4

        def mark(step):
            if trace is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                trace.append((step, ev))

        mark("start")
        if self.exchange == "p2p":
            # every phase writes into the other ranks' buffers: all ranks must
            # have finished the previous phase (and the previous execution)
            for k in (0, *mids, last):
                self._barrier()
                mark("barrier")
                self.phases.phase(k, x if k == 0 else None, out if k == last else None)
                mark(f"phase{k}")
            return out
        a, b = self._buffers()
        self.phases.phase(0, x, a)
        mark("phase0")
        cur = self._exchange(a, b)
        mark("exchange")
        for k in mids:
            dst = a if cur is b else b
            self.phases.phase(k, cur, dst)
            mark(f"phase{k}")
            other = b if dst is a else a
            cur = self._exchange(dst, other)
            mark("exchange")
        self.phases.phase(last, cur, out)
        mark(f"phase{last}")
        return out

    __call__ = execute
