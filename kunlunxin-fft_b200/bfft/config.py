"""Configuration loading and run manifests (host-only, no torch import).

B200 counterpart of the reference's ``src/xpu/config.py``: the same loaders,
dataclasses, taxonomy and hashing, reading this package's ``config/`` tree
(the B200 device profile, the B200 design space and the B200 size lists).
``DeviceProfile.hash()`` is the ``profile_hash`` the selector table is bound
to (reference: ``src/xpu/config.py:55-95``).
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
from dataclasses import asdict, dataclass, field

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CONFIG_DIR = os.path.join(_ROOT, "config")


class ConfigError(ValueError):
    """A config file is missing, unreadable, or fails its schema."""


# Semantic key taxonomy (reference: src/xpu/config.py:34-36).  The selector's
# exact key is (transform_type, transform_direction, normalization, direction,
# N, batch) inside one (device, profile_hash, precision, env) table.
TRANSFORM_TYPES = ("c2c", "r2c", "c2r")
TRANSFORM_DIRECTIONS = ("forward", "inverse")
NORMALIZATIONS = ("none", "forward", "backward", "ortho")


def read_config(name: str, config_dir: str | None = None) -> dict:
    path = os.path.join(config_dir or CONFIG_DIR, name)
    if not os.path.exists(path):
        raise ConfigError(f"missing config file: {path}")
    with open(path) as f:
        try:
            return json.load(f)
        except json.JSONDecodeError as e:
            raise ConfigError(f"{path} is not valid JSON: {e}") from e


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ConfigError(msg)


def _pow2_list(vals) -> bool:
    return (isinstance(vals, list) and bool(vals)
            and all(isinstance(v, int) and v > 0 and (v & (v - 1)) == 0 for v in vals))


@dataclass(frozen=True)
class DeviceProfile:
    """Validated B200 hardware profile (config/device.json)."""

    device: str
    board: str
    driver: str
    sm_arch: int
    sms: int
    max_threads_per_sm: int
    shared_mem_bytes: int
    hbm_gib: int
    device_code_path: str
    torch_device_key: str
    baseline: str
    vendor_fft_max_n: int

    _STR = ("device", "board", "driver", "device_code_path", "torch_device_key", "baseline")
    _INT = ("sm_arch", "sms", "max_threads_per_sm", "shared_mem_bytes", "hbm_gib",
            "vendor_fft_max_n")

    @staticmethod
    def load(config_dir: str | None = None) -> "DeviceProfile":
        d = read_config("device.json", config_dir)
        for key in DeviceProfile._STR:
            _require(isinstance(d.get(key), str) and d[key],
                     f"device.json: {key} must be a non-empty string")
        for key in DeviceProfile._INT:
            _require(isinstance(d.get(key), int) and d[key] > 0,
                     f"device.json: {key} must be a positive int")
        return DeviceProfile(**{k: d[k] for k in DeviceProfile._STR + DeviceProfile._INT})

    def hash(self) -> str:
        """16-hex sha256 of the profile fields (the table's profile_hash)."""
        blob = json.dumps(asdict(self), sort_keys=True).encode()
        return hashlib.sha256(blob).hexdigest()[:16]

    # Reference field names (src/xpu/config.py:58-69) kept as read-only aliases.
    @property
    def xpu_arch(self) -> int:
        return self.sm_arch

    @property
    def clusters(self) -> int:
        return self.sms


@dataclass(frozen=True)
class SizeMatrix:
    """Validated length lists (config/sizes.json)."""

    correctness_sizes: tuple
    bench_sizes: tuple
    blocksizes: tuple
    vendor_baseline_max_n: int

    @staticmethod
    def load(config_dir: str | None = None) -> "SizeMatrix":
        d = read_config("sizes.json", config_dir)
        for key in ("correctness_sizes", "bench_sizes", "blocksizes"):
            _require(_pow2_list(d.get(key)), f"sizes.json: {key} must be a non-empty list of powers of two")
        _require(isinstance(d.get("vendor_baseline_max_n"), int),
                 "sizes.json: vendor_baseline_max_n must be an int")
        return SizeMatrix(tuple(d["correctness_sizes"]), tuple(d["bench_sizes"]),
                          tuple(d["blocksizes"]), d["vendor_baseline_max_n"])


@dataclass(frozen=True)
class DesignSpace:
    """Validated design space (config/butterfly_space.json).

    Same axes as the reference's P800 space (src/xpu/config.py:98-265); the B200
    values differ: matrix / fused tiles reach the CTA-resident limit of the pass
    kernel (4096 points), the batch axis covers every power of two a table may
    key on, and the internal layout is interleaved complex64.
    """

    space_id: str
    target: str
    radix: tuple
    dit_bitrev_input_fold: tuple
    dif_bitrev_output_fold: tuple
    fused_tile_candidates: tuple
    batch_candidates: tuple
    batch_variants: tuple
    layout_in: str
    layout_out: str
    matrix_tiles: tuple
    matrix_rows: tuple
    matrix_default: tuple | None
    grouped_tiles: tuple
    grouped_rows: tuple
    grouped_glog: tuple
    grouped_maxp: tuple
    grouped_cells: tuple
    hybrid_tiles: tuple

    @staticmethod
    def load(config_dir: str | None = None) -> "DesignSpace":
        d = read_config("butterfly_space.json", config_dir)
        _require(isinstance(d.get("space_id"), str) and d["space_id"], "butterfly_space.json: space_id required")
        _require(isinstance(d.get("target"), str) and d["target"], "butterfly_space.json: target required")
        p = d.get("P", {})
        _require(isinstance(p.get("radix"), list) and p["radix"], "butterfly_space.json: P.radix required")
        dit = p.get("dit_stage_kernel", {})
        dif = p.get("dif_stage_kernel", {})
        _require(isinstance(dit.get("bitrev_input_fold"), list),
                 "butterfly_space.json: P.dit_stage_kernel.bitrev_input_fold required")
        _require(isinstance(dif.get("bitrev_output_fold"), list),
                 "butterfly_space.json: P.dif_stage_kernel.bitrev_output_fold required")
        tiles = p.get("stage_fusion", {}).get("fused_tiles", [1])
        _require(_pow2_list(tiles), "butterfly_space.json: P.stage_fusion.fused_tiles must be powers of two")
        batch = p.get("batch_expansion", {})
        bc = batch.get("candidates", [1])
        _require(_pow2_list(bc), "butterfly_space.json: P.batch_expansion.candidates must be powers of two")
        bv = batch.get("variants", [])
        _require(isinstance(bv, list) and all(v in ("spread", "folded") for v in bv),
                 "butterfly_space.json: P.batch_expansion.variants must be 'spread'/'folded'")
        reg = p.get("register_matrix")
        _require(isinstance(reg, dict), "butterfly_space.json: P.register_matrix required")
        for name in ("tiles", "rows"):
            _require(_pow2_list(reg.get(name)), f"butterfly_space.json: P.register_matrix.{name} must be powers of two")
        md = None
        if reg.get("default") is not None:
            rd = reg["default"]
            _require(isinstance(rd, dict) and rd.get("tile") in reg["tiles"] and rd.get("rows") in reg["rows"],
                     "butterfly_space.json: P.register_matrix.default must pick tile/rows from the published lists")
            md = (int(rd["tile"]), int(rd["rows"]))
        grp = p.get("grouped_boundary")
        _require(isinstance(grp, dict), "butterfly_space.json: P.grouped_boundary required")
        for name in ("tiles", "rows", "maxp", "cells"):
            _require(_pow2_list(grp.get(name)), f"butterfly_space.json: P.grouped_boundary.{name} must be powers of two")
        glog = grp.get("glog")
        _require(isinstance(glog, list) and glog and all(isinstance(g, int) and g >= 1 for g in glog),
                 "butterfly_space.json: P.grouped_boundary.glog must be ints >= 1")
        hyb = p.get("hybrid", {}).get("tiles", [64])
        _require(_pow2_list(hyb), "butterfly_space.json: P.hybrid.tiles must be powers of two")
        lay = d.get("L", {})
        _require(isinstance(lay.get("in"), list) and lay["in"], "butterfly_space.json: L.in required")
        _require(isinstance(lay.get("out"), list) and lay["out"], "butterfly_space.json: L.out required")
        return DesignSpace(
            space_id=d["space_id"], target=d["target"], radix=tuple(p["radix"]),
            dit_bitrev_input_fold=tuple(dit["bitrev_input_fold"]),
            dif_bitrev_output_fold=tuple(dif["bitrev_output_fold"]),
            fused_tile_candidates=tuple(tiles), batch_candidates=tuple(bc), batch_variants=tuple(bv),
            layout_in=lay["in"][0], layout_out=lay["out"][0],
            matrix_tiles=tuple(reg["tiles"]), matrix_rows=tuple(reg["rows"]), matrix_default=md,
            grouped_tiles=tuple(grp["tiles"]), grouped_rows=tuple(grp["rows"]),
            grouped_glog=tuple(glog), grouped_maxp=tuple(grp["maxp"]), grouped_cells=tuple(grp["cells"]),
            hybrid_tiles=tuple(hyb),
        )


def git_commit() -> str:
    """Best-effort current commit hash; 'unknown' outside a repository."""
    try:
        out = subprocess.run(["git", "rev-parse", "HEAD"], cwd=_ROOT, capture_output=True,
                             text=True, timeout=10)
        return out.stdout.strip() or "unknown"
    except Exception:  # noqa: BLE001
        return "unknown"


def git_dirty() -> bool:
    """True when tracked files differ from HEAD (untracked output is ignored)."""
    try:
        out = subprocess.run(["git", "status", "--porcelain", "--untracked-files=no"], cwd=_ROOT,
                             capture_output=True, text=True, timeout=10)
        return bool(out.stdout.strip())
    except Exception:  # noqa: BLE001
        return False


@dataclass
class Manifest:
    """Per-run provenance record (reference: src/xpu/config.py:302-335)."""

    commit: str
    dirty: bool
    profile_hash: str
    device: str
    driver: str
    sm_arch: int
    torch_device_key: str
    dtype: str = "complex64"
    direction: str = "forward"
    precision: str = "fp32"
    flow_id: str = "baseline-global-stage"
    processing_unit: str = "radix2-scalar"
    us: int = 1
    ts: int = 1
    ud: int = 1
    td: int = 1
    boundary_residence: str = "gm"
    layout: str = "interleaved-c64"
    block: int = 256
    fused_tile: int = 1
    warmup: int = 10
    trials: int = 50
    correctness_threshold: float = 1e-4
    command: str = ""
    extra: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


def build_manifest(profile: DeviceProfile, **overrides) -> Manifest:
    """Manifest pinned to the current commit and profile."""
    m = Manifest(commit=git_commit(), dirty=git_dirty(), profile_hash=profile.hash(),
                 device=profile.device, driver=profile.driver, sm_arch=profile.sm_arch,
                 torch_device_key=profile.torch_device_key)
    for k, v in overrides.items():
        if not hasattr(m, k):
            raise ConfigError(f"unknown manifest field: {k}")
        setattr(m, k, v)
    return m
