"""Build of the CUDA library libbfft.so (nvcc, sm_100a, in-tree).

``build()`` compiles ``csrc/*.cu`` into ``bfft/_lib/libbfft.so`` with
``-gencode arch=compute_100a,code=sm_100a`` and records the compiler version
in ``bfft/_lib/build_meta.json`` (part of the environment fingerprint).  The
library is linked against the static CUDA runtime and carries no torch
dependency; the Python layer loads it with ctypes.
"""
from __future__ import annotations

import glob
import hashlib
import json
import os
import re
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libbfft.so")
META_PATH = os.path.join(LIB_DIR, "build_meta.json")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-Wall"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + \
        sorted(glob.glob(os.path.join(INCLUDE, "*.h")))


def source_hash() -> str:
    h = hashlib.sha256()
    for p in _deps():
        with open(p, "rb") as f:
            h.update(os.path.basename(p).encode())
            h.update(f.read())
    return h.hexdigest()[:16]


def build_meta() -> dict | None:
    try:
        with open(META_PATH) as f:
            return json.load(f)
    except (OSError, json.JSONDecodeError):
        return None


def up_to_date() -> bool:
    meta = build_meta()
    return os.path.exists(LIB_PATH) and meta is not None and meta.get("source_hash") == source_hash()


def build(force: bool = False, verbose: bool = True) -> str:
    """Compile libbfft.so if its sources changed; returns the library path."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, *sources()]
    if verbose:
        print("[bfft] " + " ".join(cmd), file=sys.stderr, flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    ver = subprocess.run([nvcc, "--version"], capture_output=True, text=True).stdout
    m = re.search(r"release ([0-9.]+), V([0-9.]+)", ver)
    meta = {"nvcc": m.group(2) if m else ver.strip().splitlines()[-1],
            "arch": "sm_100a", "flags": ARCH_FLAGS + NVCC_FLAGS, "source_hash": source_hash()}
    with open(META_PATH, "w") as f:
        json.dump(meta, f, indent=1)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv)
