"""Live environment fingerprint of the CUDA stack (``env_hash``).

Reference behaviour (src/xpu/envcheck.py:1-103): gather what identifies the
device *family* and the software stack; anything missing makes the whole
fingerprint unknown (``None``) and callers fail closed (the selector abstains to
M0).  On B200 the fingerprint is the driver version, the torch and CUDA runtime
versions, the nvcc that built libbfft, the device name, SM count and the
opt-in shared memory per block.  No per-card identity (UUID, bus id) is
included: same-model cards on the same stack share one ``env_hash``.
"""
from __future__ import annotations

import hashlib
import json
from functools import lru_cache

_REQUIRED = ("driver", "torch", "cuda_runtime", "nvcc", "device_name", "multiprocessor_count",
             "max_shared_mem_optin", "compute_capability")

SCOPE = "card-family"


def _driver_version() -> str | None:
    try:
        import pynvml  # nvidia-ml-py

        pynvml.nvmlInit()
        try:
            v = pynvml.nvmlSystemGetDriverVersion()
            return v.decode() if isinstance(v, bytes) else str(v)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # noqa: BLE001
        return None


def _nvcc_version() -> str | None:
    try:
        from . import _build

        meta = _build.build_meta()
        return meta.get("nvcc") if meta else None
    except Exception:  # noqa: BLE001
        return None


@lru_cache(maxsize=4)
def collect(device: int = 0) -> dict | None:
    """Best-effort live fingerprint of ``device``; ``None`` = unknown."""
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        props = torch.cuda.get_device_properties(device)
        env = {
            "torch": torch.__version__,
            "cuda_runtime": torch.version.cuda,
            "driver": _driver_version(),
            "nvcc": _nvcc_version(),
            "device_name": props.name,
            "multiprocessor_count": int(props.multi_processor_count),
            "max_shared_mem_optin": int(getattr(props, "shared_memory_per_block_optin", 0)) or None,
            "compute_capability": f"{props.major}.{props.minor}",
        }
    except Exception:  # noqa: BLE001
        return None
    if any(env.get(k) in (None, "") for k in _REQUIRED):
        return None
    return env


def env_hash(env: dict | None = None) -> str | None:
    """16-hex hash of a fingerprint dict; ``None`` when it is unknown."""
    if env is None:
        env = collect()
    if env is None:
        return None
    blob = json.dumps(env, sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(blob.encode()).hexdigest()[:16]


def current_env_hash() -> str | None:
    return env_hash(collect())
