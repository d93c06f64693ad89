"""ctypes binding of libbfft.so (the C ABI declared in include/bfft.h).

The Python layer reaches the GPU only through these entry points.  There is
no fallback: if the library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
import weakref

from . import _build

OK, ERR_VALUE, ERR_SHAPE, ERR_UNSUPPORTED, ERR_CUDA, ERR_NCCL, ERR_ALLOC, ERR_WORKSPACE = range(8)

RUNNER_IDS = {
    "fft_dit": 0, "fft_dif": 1, "fft_dit_batch": 2, "fft_dif_batch": 3,
    "fft_dit_radix4": 4, "fft_dif_radix4": 5, "fft_dit_radix4_batch": 6, "fft_dif_radix4_batch": 7,
    "fft_dit_fused": 8, "fft_dit_matrix": 9, "fft_dif_matrix": 10, "fft_dit_matrix_batch": 11,
    "fft_dif_matrix_batch": 12, "fft_dit_grouped": 13, "fft_dif_grouped": 14, "run_hybrid": 15,
}
TRANSFORM_TYPE_IDS = {"c2c": 0, "r2c": 1, "c2r": 2}
TRANSFORM_DIRECTION_IDS = {"forward": 0, "inverse": 1}
NORM_IDS = {"none": 0, "forward": 1, "backward": 2, "ortho": 3}
VARIANT_IDS = {"spread": 0, "folded": 1}

# Every symbol include/bfft.h declares.
EXPORTS = ("bfft_api_version", "bfft_last_error", "bfft_plan_create", "bfft_plan_workspace_size",
           "bfft_plan_launches", "bfft_execute", "bfft_plan_destroy", "bfft_bit_reverse_permute",
           "bfft_r2c_stitch", "bfft_c2r_pre", "bfft_c2r_unpack", "bfft_twiddle_table",
           "bfft_index_map", "bfft_launch_counter", "bfft_hybrid_c2c_noalloc", "bfft_tc_dft16_rows",
           "bfft_dist_batch_shard", "bfft_dist_plan_create", "bfft_dist_workspace_size",
           "bfft_dist_phase", "bfft_dist_plan_launches", "bfft_dist_plan_destroy", "bfft_device_status",
           "bfft_probe_bounded_waits",
           "bfft_stream_plan_create", "bfft_stream_plan_info", "bfft_stream_execute", "bfft_stream_plan_destroy",
           "bfft_dist_p2p_prepare", "bfft_dist_p2p_attach", "bfft_dist_p2p_attach_pointers", "bfft_dist_p2p_phase")


class PlanDesc(ctypes.Structure):
    """Mirror of struct bfft_plan_desc."""

    _fields_ = [("runner", ctypes.c_int32), ("direction", ctypes.c_int32),
                ("n", ctypes.c_int64), ("batch", ctypes.c_int64),
                ("transform_type", ctypes.c_int32), ("transform_direction", ctypes.c_int32),
                ("norm", ctypes.c_int32), ("real_flow", ctypes.c_int32),
                ("block", ctypes.c_int32), ("tile", ctypes.c_int32), ("rows", ctypes.c_int32),
                ("glog", ctypes.c_int32), ("maxp", ctypes.c_int32), ("cells", ctypes.c_int32),
                ("variant", ctypes.c_int32), ("device", ctypes.c_int32)]


_lib = None
_lock = threading.Lock()


def library_path() -> str:
    return _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load libbfft.so (raises RuntimeError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not os.path.exists(path):
            raise RuntimeError(f"libbfft.so not found at {path}; build it with "
                               "bfft._build.build() (nvcc, sm_100a) -- there is no CPU fallback")
        L = ctypes.CDLL(path)
        vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t
        L.bfft_api_version.restype = ctypes.c_int
        L.bfft_last_error.restype = ctypes.c_char_p
        L.bfft_launch_counter.restype = ctypes.c_uint64
        L.bfft_plan_create.argtypes = [ctypes.POINTER(PlanDesc), ctypes.POINTER(vp)]
        L.bfft_plan_workspace_size.argtypes = [vp, ctypes.POINTER(sz)]
        L.bfft_plan_launches.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        L.bfft_execute.argtypes = [vp, vp, vp, vp, sz, vp]
        L.bfft_plan_destroy.argtypes = [vp]
        L.bfft_bit_reverse_permute.argtypes = [vp, vp, i64, i64, i32, vp]
        L.bfft_r2c_stitch.argtypes = [vp, vp, i64, i64, ctypes.c_float, i32, vp]
        L.bfft_c2r_pre.argtypes = [vp, vp, i64, i64, i32, vp]
        L.bfft_c2r_unpack.argtypes = [vp, vp, i64, i64, ctypes.c_float, i32, vp]
        L.bfft_twiddle_table.argtypes = [vp, i64, i64, i32, vp]
        L.bfft_index_map.argtypes = [i32, i32, vp, i32, vp]
        L.bfft_hybrid_c2c_noalloc.argtypes = [vp, vp, i64, i64, i64, i32, i32, i32, vp]
        L.bfft_tc_dft16_rows.argtypes = [vp, vp, i64, i32, ctypes.c_float, i32, vp]
        L.bfft_dist_batch_shard.argtypes = [i64, i32, i32, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.bfft_dist_plan_create.argtypes = [i64, i64, i32, i32, i32, i32, i32, i32, i32, ctypes.POINTER(vp)]
        L.bfft_dist_workspace_size.argtypes = [vp, ctypes.POINTER(sz)]
        L.bfft_dist_phase.argtypes = [vp, i32, vp, vp, vp, sz, vp]
        L.bfft_dist_plan_launches.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int)]
        L.bfft_dist_plan_destroy.argtypes = [vp]
        L.bfft_device_status.argtypes = [i32, ctypes.POINTER(ctypes.c_uint32), i32]
        L.bfft_probe_bounded_waits.argtypes = [i32, vp]
        L.bfft_stream_plan_create.argtypes = [ctypes.POINTER(PlanDesc), i64, ctypes.POINTER(vp)]
        L.bfft_stream_plan_info.argtypes = [vp, ctypes.POINTER(sz), ctypes.POINTER(sz), ctypes.POINTER(ctypes.c_int)]
        L.bfft_stream_execute.argtypes = [vp, vp, vp, vp]
        L.bfft_stream_plan_destroy.argtypes = [vp]
        L.bfft_dist_p2p_prepare.argtypes = [vp, ctypes.POINTER(vp), ctypes.c_char_p, ctypes.POINTER(sz)]
        L.bfft_dist_p2p_attach.argtypes = [vp, ctypes.c_char_p]
        L.bfft_dist_p2p_attach_pointers.argtypes = [vp, ctypes.POINTER(vp)]
        L.bfft_dist_p2p_phase.argtypes = [vp, i32, vp, vp, vp, sz, vp]
        for name in EXPORTS:
            fn = getattr(L, name)
            if name not in ("bfft_api_version", "bfft_last_error", "bfft_launch_counter"):
                fn.restype = ctypes.c_int
        _lib = L
        return L


def last_error() -> str:
    msg = load().bfft_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(status: int, what: str = "bfft") -> None:
    """Map a bfft_status onto the reference's exception types."""
    if status == OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (ERR_VALUE, ERR_SHAPE, ERR_UNSUPPORTED, ERR_WORKSPACE):
        raise ValueError(msg)
    if status == ERR_ALLOC:
        raise MemoryError(msg)
    raise RuntimeError(msg)


def device_status(device: int = 0, clear: bool = False) -> int:
    """Status bits the kernels set when a bounded wait expired (0 = healthy)."""
    v = ctypes.c_uint32()
    check(load().bfft_device_status(int(device), ctypes.byref(v), 1 if clear else 0), "bfft_device_status")
    return int(v.value)


def launch_counter() -> int:
    return int(load().bfft_launch_counter())


def _destroy(handle: int) -> None:
    try:
        if _lib is not None and handle:
            _lib.bfft_plan_destroy(ctypes.c_void_p(handle))
    except Exception:  # noqa: BLE001 - interpreter shutdown
        pass


class NativePlan:
    """Owns one bfft_plan_t; destroyed with the Python object."""

    def __init__(self, desc: PlanDesc):
        L = load()
        h = ctypes.c_void_p()
        check(L.bfft_plan_create(ctypes.byref(desc), ctypes.byref(h)), "bfft_plan_create")
        self.handle = h.value
        self.desc = desc
        ws = ctypes.c_size_t()
        check(L.bfft_plan_workspace_size(self.handle, ctypes.byref(ws)), "bfft_plan_workspace_size")
        self.workspace_bytes = int(ws.value)
        nl = ctypes.c_int()
        check(L.bfft_plan_launches(self.handle, ctypes.byref(nl)), "bfft_plan_launches")
        self.launches = int(nl.value)
        self._fin = weakref.finalize(self, _destroy, self.handle)

    def execute(self, in_ptr: int, out_ptr: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
        check(load().bfft_execute(self.handle, in_ptr, out_ptr, ws_ptr, ws_bytes, stream),
              "bfft_execute")


def _destroy_dist(handle: int) -> None:
    try:
        if _lib is not None and handle:
            _lib.bfft_dist_plan_destroy(ctypes.c_void_p(handle))
    except Exception:  # noqa: BLE001 - interpreter shutdown
        pass


class NativeDistPlan:
    """Owns one bfft_dist_plan_t (the device phases of the distributed 4-step)."""

    def __init__(self, n1: int, n2: int, nranks: int, rank: int, *, transform_direction: str = "forward",
                 norm: str = "backward", row_tiles: tuple[int, int] = (0, 0), device: int = 0):
        L = load()
        h = ctypes.c_void_p()
        check(L.bfft_dist_plan_create(int(n1), int(n2), int(nranks), int(rank),
                                      TRANSFORM_DIRECTION_IDS[transform_direction], NORM_IDS[norm],
                                      int(row_tiles[0]), int(row_tiles[1]), int(device), ctypes.byref(h)),
              "bfft_dist_plan_create")
        self.handle = h.value
        ws = ctypes.c_size_t()
        check(L.bfft_dist_workspace_size(self.handle, ctypes.byref(ws)), "bfft_dist_workspace_size")
        self.workspace_bytes = int(ws.value)
        self.launches = []  # per phase 0..4 (4: the transposed-output phase)
        for ph in range(5):
            nl = ctypes.c_int()
            check(L.bfft_dist_plan_launches(self.handle, ph, ctypes.byref(nl)), "bfft_dist_plan_launches")
            self.launches.append(int(nl.value))
        self._fin = weakref.finalize(self, _destroy_dist, self.handle)

    def phase(self, phase: int, in_ptr: int, out_ptr: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
        check(load().bfft_dist_phase(self.handle, int(phase), in_ptr, out_ptr, ws_ptr, ws_bytes, stream),
              "bfft_dist_phase")

    # ---- peer-to-peer mode ----
    def p2p_prepare(self) -> tuple[int, bytes]:
        """(device address of this rank's exchange buffers, its CUDA IPC handle)."""
        base, n = ctypes.c_void_p(), ctypes.c_size_t()
        check(load().bfft_dist_p2p_prepare(self.handle, ctypes.byref(base), None, ctypes.byref(n)),
              "bfft_dist_p2p_prepare")
        buf = ctypes.create_string_buffer(int(n.value))
        check(load().bfft_dist_p2p_prepare(self.handle, None, buf, ctypes.byref(n)), "bfft_dist_p2p_prepare")
        return int(base.value), buf.raw

    def p2p_attach(self, handles: bytes) -> None:
        check(load().bfft_dist_p2p_attach(self.handle, handles), "bfft_dist_p2p_attach")

    def p2p_attach_pointers(self, bases: list[int]) -> None:
        arr = (ctypes.c_void_p * len(bases))(*bases)
        check(load().bfft_dist_p2p_attach_pointers(self.handle, arr), "bfft_dist_p2p_attach_pointers")

    def p2p_phase(self, phase: int, in_ptr: int, out_ptr: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
        check(load().bfft_dist_p2p_phase(self.handle, int(phase), in_ptr, out_ptr, ws_ptr, ws_bytes, stream),
              "bfft_dist_p2p_phase")


def _destroy_stream(handle: int) -> None:
    try:
        if _lib is not None and handle:
            _lib.bfft_stream_plan_destroy(ctypes.c_void_p(handle))
    except Exception:  # noqa: BLE001 - interpreter shutdown
        pass


class NativeStreamPlan:
    """Owns one bfft_stream_plan_t (host-to-host pipelined execution)."""

    def __init__(self, chunk_desc: PlanDesc, chunks: int):
        L = load()
        h = ctypes.c_void_p()
        check(L.bfft_stream_plan_create(ctypes.byref(chunk_desc), int(chunks), ctypes.byref(h)),
              "bfft_stream_plan_create")
        self.handle = h.value
        self.chunks = int(chunks)
        ib, ob, nl = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int()
        check(L.bfft_stream_plan_info(self.handle, ctypes.byref(ib), ctypes.byref(ob), ctypes.byref(nl)),
              "bfft_stream_plan_info")
        self.in_bytes, self.out_bytes, self.launches_per_chunk = int(ib.value), int(ob.value), int(nl.value)
        self._fin = weakref.finalize(self, _destroy_stream, self.handle)

    def execute(self, host_in: int, host_out: int, stream: int) -> None:
        check(load().bfft_stream_execute(self.handle, host_in, host_out, stream), "bfft_stream_execute")


def batch_shard(batch: int, nranks: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank` in a batch split over `nranks` (bfft_dist_batch_shard)."""
    first, count = ctypes.c_int64(), ctypes.c_int64()
    check(load().bfft_dist_batch_shard(int(batch), int(nranks), int(rank), ctypes.byref(first),
                                       ctypes.byref(count)), "bfft_dist_batch_shard")
    return int(first.value), int(count.value)


def make_desc(runner: str, direction: str, n: int, batch: int, *, transform_type: str = "c2c",
              transform_direction: str = "forward", norm: str = "backward", real_flow: bool = False,
              block: int = 256, tile: int = 0, rows: int = 0, glog: int = 2, maxp: int = 4096,
              cells: int = 1, variant: str = "spread", device: int = 0) -> PlanDesc:
    if runner not in RUNNER_IDS:
        raise ValueError(f"unknown runner {runner!r}")
    if variant not in VARIANT_IDS:
        raise ValueError(f"variant must be 'spread' or 'folded', got {variant!r}")
    return PlanDesc(runner=RUNNER_IDS[runner], direction=0 if direction == "dit" else 1, n=int(n),
                    batch=int(batch), transform_type=TRANSFORM_TYPE_IDS[transform_type],
                    transform_direction=TRANSFORM_DIRECTION_IDS[transform_direction],
                    norm=NORM_IDS[norm], real_flow=1 if real_flow else 0, block=int(block),
                    tile=int(tile), rows=int(rows), glog=int(glog), maxp=int(maxp),
                    cells=int(cells), variant=VARIANT_IDS[variant], device=int(device))
