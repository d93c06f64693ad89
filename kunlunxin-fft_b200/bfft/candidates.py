"""Lowering contract for selector-table entries (host-only, no torch).

The reference checks every table entry against the lowering its P800 Triton
backend accepts (src/xpu/candidates.py:189-383) before the table may be used.
This module applies the same contract to the B200 lowerings: the same schema-v2
attribution axes (flow_id / flow_realization / processing_unit /
local_residence), the same knob rules, with the B200 internal layout
(interleaved complex64) in place of the P800 planar split.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

from .config import DeviceProfile
from .semantic import SPECIALIZED_FLOWS

SPECIALIZED_ROUTING = frozenset().union(*SPECIALIZED_FLOWS.values())

_LOCAL_FLOWS = frozenset({"local-fused-tile"})
_GLOBAL_CORE_FLOWS = frozenset({"baseline-global-stage", "batch-spread", "batch-folded"})
_BATCH_SPREAD_FLOWS = frozenset({"batch-spread"})

PROCESSING_UNITS = ("radix2-scalar", "radix4-scalar", "dense-dot-fft64", "composite-linear-map")
UNIT_RADIX = {"radix2-scalar": 2, "radix4-scalar": 4, "dense-dot-fft64": 2, "composite-linear-map": 2}
FLOW_REALIZATIONS = ("global-stage", "fused-inplace", "matrix-resident", "grouped-boundary")
REALIZATION_UNITS = {
    "global-stage": ("radix2-scalar", "radix4-scalar"),
    "fused-inplace": ("radix2-scalar", "radix4-scalar"),
    "matrix-resident": ("dense-dot-fft64",),
    "grouped-boundary": ("composite-linear-map",),
}
LOCAL_RESIDENCES = ("none", "cache", "register", "implicit-dot", "register+implicit-dot")
REALIZATION_LOCAL_RESIDENCES = {
    "global-stage": ("none",),
    "fused-inplace": ("none", "cache"),
    "matrix-resident": ("register", "implicit-dot", "register+implicit-dot"),
    "grouped-boundary": ("register",),
}
_DERIVED_LOCAL_RESIDENCE = {
    "global-stage": "none",
    "fused-inplace": "cache",
    "matrix-resident": "register+implicit-dot",
    "grouped-boundary": "register",
}
LAYOUT = "interleaved-c64"


class LoweringStatus:
    LEGAL = "legal"
    NOT_LOWERED = "not-lowered"
    INFEASIBLE = "infeasible"


def _is_local(flow) -> bool:
    return flow in _LOCAL_FLOWS or flow in SPECIALIZED_ROUTING


def _is_global(flow) -> bool:
    return flow in _GLOBAL_CORE_FLOWS or flow in SPECIALIZED_ROUTING


@dataclass(frozen=True)
class Candidate:
    """One point of the design space (schema v2)."""

    flow_id: str
    processing_unit: str
    radix: int
    us: int = 1
    ts: int = 1
    ud: int = 1
    td: int = 1
    boundary_residence: str = "gm"
    pipeline: str = "none"
    layout: str = LAYOUT
    block: int = 256
    fused_tile: int = 1
    dit_bitrev_input_fold: bool = True
    dif_bitrev_output_fold: bool = True
    batch: int = 1
    batch_variant: str = "none"
    flow_realization: str = ""
    local_residence: str = ""
    rows: int = 1
    glog: int = 0
    maxp: int = 0
    cells: int = 1

    def to_dict(self) -> dict:
        d = asdict(self)
        d["flow_realization"] = effective_flow_realization(self)
        d["local_residence"] = effective_local_residence(self)
        return d


def effective_flow_realization(c: Candidate) -> str:
    if c.flow_realization:
        return c.flow_realization
    if c.flow_id in _GLOBAL_CORE_FLOWS:
        return "global-stage"
    if c.glog >= 1:
        return "grouped-boundary"
    if c.rows > 1:
        return "matrix-resident"
    return "fused-inplace"


def effective_local_residence(c: Candidate) -> str:
    return c.local_residence or _DERIVED_LOCAL_RESIDENCE[effective_flow_realization(c)]


@dataclass(frozen=True)
class Verdict:
    candidate: Candidate
    status: str
    reasons: tuple = ()

    @property
    def legal(self) -> bool:
        return self.status == LoweringStatus.LEGAL

    def to_dict(self) -> dict:
        return {"candidate": self.candidate.to_dict(), "status": self.status,
                "reasons": list(self.reasons)}


def _pow2(name: str, val: int, reasons: list, minimum: int = 1) -> None:
    if val < minimum or (val & (val - 1)) != 0:
        reasons.append(f"{name}: must be a power of two >= {minimum}, got {val}")


def check_lowering(c: Candidate, profile: DeviceProfile | None = None) -> Verdict:
    """Apply the B200 lowering contract; rejections carry their reasons."""
    reasons: list[str] = []
    real = effective_flow_realization(c)
    local_res = effective_local_residence(c)

    if c.processing_unit not in UNIT_RADIX:
        reasons.append(f"processing-unit: only {', '.join(PROCESSING_UNITS)} are implemented; "
                       f"{c.processing_unit!r} is not-lowered")
    elif c.radix not in (2, 4):
        reasons.append(f"radix: must be 2 or 4, got {c.radix}")
    elif c.radix != UNIT_RADIX[c.processing_unit]:
        reasons.append(f"processing-unit: {c.processing_unit!r} must match "
                       f"radix={UNIT_RADIX[c.processing_unit]} (got radix={c.radix})")

    if c.layout != LAYOUT:
        reasons.append(f"layout: the B200 lowering accepts {LAYOUT!r}, got {c.layout!r}")
    if c.boundary_residence != "gm":
        reasons.append("boundary_residence: passes exchange through device memory ('gm'); "
                       f"got {c.boundary_residence!r}")

    _pow2("block", c.block, reasons)
    _pow2("fused_tile", c.fused_tile, reasons)
    _pow2("rows", c.rows, reasons)
    _pow2("cells", c.cells, reasons)
    if c.maxp != 0:
        _pow2("maxp", c.maxp, reasons)
    if c.glog < 0:
        reasons.append(f"glog: must be >= 0, got {c.glog}")

    if real not in FLOW_REALIZATIONS:
        reasons.append(f"flow_realization: must be one of {', '.join(FLOW_REALIZATIONS)}, got {real!r}")
    else:
        local = real != "global-stage"
        if local and not _is_local(c.flow_id):
            reasons.append(f"flow_realization: {real!r} requires flow 'local-fused-tile', got {c.flow_id!r}")
        if not local and not _is_global(c.flow_id):
            reasons.append(f"flow_realization: 'global-stage' requires the baseline or a batch flow, "
                           f"got {c.flow_id!r}")
        units = REALIZATION_UNITS.get(real, ())
        if units and c.processing_unit not in units:
            reasons.append(f"processing-unit: realization {real!r} lowers only as {', '.join(units)}; "
                           f"got {c.processing_unit!r}")
        res = REALIZATION_LOCAL_RESIDENCES.get(real, ())
        if res and local_res not in res:
            reasons.append(f"local_residence: realization {real!r} evidences only {', '.join(res)}; "
                           f"got {local_res!r}")
        if real == "grouped-boundary" and c.glog < 1:
            reasons.append(f"glog: realization 'grouped-boundary' needs glog >= 1, got {c.glog}")

    if c.fused_tile > 1 and not _is_local(c.flow_id):
        reasons.append(f"flow_id: fused_tile={c.fused_tile} requires flow 'local-fused-tile', got {c.flow_id!r}")
    if c.fused_tile == 1 and not _is_global(c.flow_id):
        reasons.append(f"flow_id: fused_tile=1 requires flow 'baseline-global-stage' or a batch flow, "
                       f"got {c.flow_id!r}")

    if c.batch_variant == "none":
        if c.batch != 1:
            reasons.append(f"batch: batch={c.batch} needs a batch variant ('spread'/'folded'); "
                           "got batch_variant='none'")
        if c.flow_id in ("batch-spread", "batch-folded"):
            reasons.append(f"flow_id: {c.flow_id!r} requires batch_variant "
                           f"'{c.flow_id.removeprefix('batch-')}', got 'none'")
        if c.ud != 1 or c.td != 1:
            reasons.append(f"data expansion: Ud/Td != 1 is lowered only through a batch variant; "
                           f"got Ud={c.ud}, Td={c.td}")
    else:
        if c.batch_variant not in ("spread", "folded"):
            reasons.append(f"batch_variant: must be 'none'/'spread'/'folded', got {c.batch_variant!r}")
            return Verdict(c, LoweringStatus.NOT_LOWERED, tuple(reasons))
        if c.batch <= 0 or (c.batch & (c.batch - 1)) != 0:
            reasons.append(f"batch: must be a power of two, got {c.batch}")
        if c.batch_variant == "spread":
            if real == "matrix-resident":
                if not _is_local(c.flow_id):
                    reasons.append(f"flow_id: matrix-resident batch keeps 'local-fused-tile', got {c.flow_id!r}")
            elif not (c.flow_id in _BATCH_SPREAD_FLOWS or c.flow_id in SPECIALIZED_ROUTING):
                reasons.append(f"flow_id: spread variant requires 'batch-spread' for {real!r}, got {c.flow_id!r}")
            if c.ud != c.batch or c.td != 1:
                reasons.append(f"data expansion: spread requires Ud=batch={c.batch}, Td=1; "
                               f"got Ud={c.ud}, Td={c.td}")
        else:
            if real != "global-stage" or c.processing_unit != "radix2-scalar":
                reasons.append(f"batch_variant: folded (Td) lowers the M4 radix-2 stage cascade only; "
                               f"{real}/{c.processing_unit} folded is not-lowered")
            elif c.flow_id != "batch-folded":
                reasons.append(f"flow_id: folded variant requires 'batch-folded', got {c.flow_id!r}")
            if c.ud != 1 or c.td != c.batch:
                reasons.append(f"data expansion: folded requires Ud=1, Td=batch={c.batch}; "
                               f"got Ud={c.ud}, Td={c.td}")
        if c.fused_tile > 1 and not (real == "matrix-resident" and c.batch_variant == "spread"):
            reasons.append(f"fused_tile: batched paths consume fused_tile only for the matrix-resident "
                           f"spread lowering; got fused_tile={c.fused_tile}")

    if c.pipeline != "none":
        reasons.append(f"pipeline: {c.pipeline!r} is not-lowered (no overlap evidence)")

    status = LoweringStatus.NOT_LOWERED if reasons else LoweringStatus.LEGAL
    return Verdict(c, status, tuple(reasons))
