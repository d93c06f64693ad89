"""bfft -- B200-native FFT operator library with the Kunlunxin-FFT plan API.

Host-only symbols (config, selector, composition, planning) import without
torch; runner functions and execution load lazily and require the CUDA
library ``libbfft.so`` (built by ``bfft._build.build()``).  The export list
mirrors the reference package (src/xpu/__init__.py:37-150).
"""
import importlib

from .composition import composition_select, load_composition_table  # noqa: F401
from .config import (ConfigError, DesignSpace, DeviceProfile, Manifest, SizeMatrix,  # noqa: F401
                     build_manifest, git_commit, git_dirty)
from .entry import (SUPPORTED_NORMS, SUPPORTED_TRANSFORM_DIRECTIONS, SUPPORTED_TRANSFORMS,  # noqa: F401
                    ExecutionPlan, ExecutionReport, norm_scale, plan_fft)
from .selector import Selection, load_table, select  # noqa: F401

_LAZY = {
    "execute_fft_plan": "entry",
    "run_fft": "entry",
    "bit_reverse_permute": "runner",
    "device_name": "runner",
    "device_ready": "context",
    "fft_dif": "runner",
    "fft_dit": "runner",
    "fft_dit_fused": "runner",
    "fft_dit_matrix": "runner",
    "fft_dif_matrix": "runner",
    "fft_dit_grouped": "runner",
    "fft_dif_grouped": "runner",
    "fft_dit_batch": "runner",
    "fft_dif_batch": "runner",
    "fft_dit_matrix_batch": "runner",
    "fft_dif_matrix_batch": "runner",
    "fft_dit_matrix_packet_batch": "runner",
    "fft_dit_radix4": "runner",
    "fft_dif_radix4": "runner",
    "fft_dit_radix4_batch": "runner",
    "fft_dif_radix4_batch": "runner",
    "r2c_stitch": "runner",
    "c2r_pre": "runner",
    "c2r_unpack": "runner",
    "log2_exact": "validate",
    "time_call": "runner",
    "time_call_detailed": "runner",
    "twiddle_tables": "runner",
    "xpu_context": "context",
    "validate_input": "validate",
    "plan_hybrid": "adapter_hybrid",
    "run_hybrid": "adapter_hybrid",
}

__all__ = sorted([
    "ConfigError", "DesignSpace", "DeviceProfile", "ExecutionPlan", "ExecutionReport", "Manifest",
    "SizeMatrix", "Selection", "SUPPORTED_NORMS", "SUPPORTED_TRANSFORMS",
    "SUPPORTED_TRANSFORM_DIRECTIONS", "build_manifest", "composition_select", "git_commit",
    "git_dirty", "load_composition_table", "load_table", "norm_scale", "plan_fft", "select",
    *_LAZY,
])


def __getattr__(name):
    if name in _LAZY:
        value = getattr(importlib.import_module(f".{_LAZY[name]}", __name__), name)
        globals()[name] = value
        return value
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return list(__all__)
