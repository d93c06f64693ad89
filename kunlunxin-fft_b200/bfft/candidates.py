"""What the B200 library can lower: the contract selector-table entries must meet.

A selector-table entry names a point of the design space (schema v2 axes:
flow_id, flow_realization, processing_unit, local residence, knobs).  The
reference refuses a table whose entries its own backend cannot lower
(src/xpu/candidates.py:189-386).  Here the question is what the plan
builder of this library accepts (``build_core`` in csrc/bfft_api.cu):

* ``global-stage``      -> the one-stage-per-launch cascades: radix-2
  (``k_radix2_stage``, M0 / M4, spread or folded batch) and radix-4
  (``k_radix4_stage``, M5, spread batch);
* ``fused-inplace``     -> a CTA-resident local group of ``fused_tile``
  points followed by radix-2 stages (M1, single transform);
* ``matrix-resident``   -> a CTA-resident local group plus tail passes
  (M2; the batched form is the batch local-fused core, spread batch);
* ``grouped-boundary``  -> a local group plus the grouped tail (M3, needs
  ``glog >= 1``).

The accepted combinations are data (``LOWERINGS``); ``check_lowering`` runs
an ordered list of rules over a candidate and collects one reason per broken
rule.  An entry is legal when no rule objects.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

from .config import DeviceProfile
from .semantic import SPECIALIZED_FLOWS

SPECIALIZED_ROUTING = frozenset().union(*SPECIALIZED_FLOWS.values())

LAYOUT = "interleaved-c64"  # complex64 (re, im) pairs, batch-major -- the only data layout here
PROCESSING_UNITS = ("radix2-scalar", "radix4-scalar", "dense-dot-fft64", "composite-linear-map")
UNIT_RADIX = {"radix2-scalar": 2, "radix4-scalar": 4, "dense-dot-fft64": 2, "composite-linear-map": 2}
FLOW_REALIZATIONS = ("global-stage", "fused-inplace", "matrix-resident", "grouped-boundary")
LOCAL_RESIDENCES = ("none", "cache", "register", "implicit-dot", "register+implicit-dot")

_STAGE_FLOWS = frozenset({"baseline-global-stage", "batch-spread", "batch-folded"})
_TILE_FLOWS = frozenset({"local-fused-tile"})


@dataclass(frozen=True)
class Lowering:
    """One realization as the plan builder implements it."""

    builder: str                 # what runs (for messages)
    units: tuple                 # processing units it is written for
    flows: frozenset             # flow ids that route to it (dedicated real flows route everywhere)
    residences: tuple            # local residences it evidences; the first is the derived default
    batch_variants: tuple        # 'none' = single transform
    folded_units: tuple = ()     # units whose folded batch form exists
    takes_tile: bool = False     # consumes fused_tile > 1
    needs_glog: bool = False


LOWERINGS = {
    "global-stage": Lowering("one radix-2 / radix-4 stage per launch", ("radix2-scalar", "radix4-scalar"),
                             _STAGE_FLOWS, ("none",), ("none", "spread", "folded"),
                             folded_units=("radix2-scalar",)),
    "fused-inplace": Lowering("CTA-resident local group + radix-2 stages", ("radix2-scalar", "radix4-scalar"),
                              _TILE_FLOWS, ("cache", "none"), ("none",), takes_tile=True),
    "matrix-resident": Lowering("CTA-resident local group + tail passes", ("dense-dot-fft64",), _TILE_FLOWS,
                                ("register+implicit-dot", "register", "implicit-dot"), ("none", "spread"),
                                takes_tile=True),
    "grouped-boundary": Lowering("local group + grouped tail passes", ("composite-linear-map",), _TILE_FLOWS,
                                 ("register",), ("none",), takes_tile=True, needs_glog=True),
}


class LoweringStatus:
    LEGAL = "legal"
    NOT_LOWERED = "not-lowered"
    INFEASIBLE = "infeasible"


@dataclass(frozen=True)
class Candidate:
    """One point of the design space (schema-v2 fields)."""

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
    """The declared realization, else the one the knobs imply."""
    if c.flow_realization:
        return c.flow_realization
    if c.flow_id in _STAGE_FLOWS:
        return "global-stage"
    return "grouped-boundary" if c.glog >= 1 else ("matrix-resident" if c.rows > 1 else "fused-inplace")


def effective_local_residence(c: Candidate) -> str:
    if c.local_residence:
        return c.local_residence
    low = LOWERINGS.get(effective_flow_realization(c))
    return low.residences[0] if low else "none"


@dataclass(frozen=True)
class Verdict:
    candidate: Candidate
    status: str
    reasons: tuple = ()

    @property
    def legal(self) -> bool:
        return self.status == LoweringStatus.LEGAL

    def to_dict(self) -> dict:
        return {"candidate": self.candidate.to_dict(), "status": self.status, "reasons": list(self.reasons)}


# ---------------------------------------------------------------- rules
#
# Each rule sees the candidate and its resolved lowering (None when the
# realization is unknown) and returns the reasons it objects with.

def _pow2(v) -> bool:
    return isinstance(v, int) and v >= 1 and v & (v - 1) == 0


def _routes(flow: str, allowed: frozenset) -> bool:
    return flow in allowed or flow in SPECIALIZED_ROUTING


def _rule_unit(c, low):
    if c.processing_unit not in UNIT_RADIX:
        return [f"processing-unit {c.processing_unit!r} has no B200 kernel (kernels exist for "
                f"{', '.join(PROCESSING_UNITS)})"]
    if c.radix != UNIT_RADIX[c.processing_unit]:
        return [f"processing-unit {c.processing_unit!r} runs radix {UNIT_RADIX[c.processing_unit]}, "
                f"the entry says radix {c.radix}"]
    return []


def _rule_layout(c, low):
    out = []
    if c.layout != LAYOUT:
        out.append(f"layout {c.layout!r}: the kernels read and write {LAYOUT!r} only")
    if c.boundary_residence != "gm":
        out.append(f"boundary_residence {c.boundary_residence!r}: passes hand over through device memory ('gm')")
    return out


def _rule_knobs(c, low):
    out = [f"{name} must be a power of two >= 1, got {val}"
           for name, val in (("block", c.block), ("fused_tile", c.fused_tile), ("rows", c.rows),
                             ("cells", c.cells)) if not _pow2(val)]
    if c.maxp != 0 and not _pow2(c.maxp):
        out.append(f"maxp must be 0 or a power of two, got {c.maxp}")
    if c.glog < 0:
        out.append(f"glog must be >= 0, got {c.glog}")
    return out


def _rule_realization(c, low):
    real = effective_flow_realization(c)
    if low is None:
        return [f"flow_realization {real!r} is not one of {', '.join(FLOW_REALIZATIONS)}"]
    out = []
    if not _routes(c.flow_id, low.flows):
        out.append(f"flow_realization {real!r} ({low.builder}) is reached from "
                   f"{' / '.join(sorted(low.flows))}, not from flow {c.flow_id!r}")
    if c.processing_unit in UNIT_RADIX and c.processing_unit not in low.units:
        out.append(f"processing-unit {c.processing_unit!r} is not what {real!r} runs ({', '.join(low.units)})")
    res = effective_local_residence(c)
    if res not in low.residences:
        out.append(f"local_residence {res!r} is not evidenced by {real!r} ({', '.join(low.residences)})")
    if low.needs_glog and c.glog < 1:
        out.append(f"glog {c.glog}: {real!r} groups at least one tail stage (glog >= 1)")
    return out


def _rule_tile(c, low):
    if c.fused_tile > 1 and not _routes(c.flow_id, _TILE_FLOWS):
        return [f"fused_tile {c.fused_tile} is a local-group size; flow {c.flow_id!r} has no local group"]
    if c.fused_tile == 1 and not _routes(c.flow_id, _STAGE_FLOWS):
        return [f"flow {c.flow_id!r} needs a local group (fused_tile > 1); fused_tile=1 runs only the stage flows"]
    return []


def _rule_batch(c, low):
    v = c.batch_variant
    if v == "none":
        out = []
        if c.batch != 1:
            out.append(f"batch {c.batch} needs a batch variant (spread or folded), the entry has none")
        if c.flow_id in ("batch-spread", "batch-folded"):
            out.append(f"flow {c.flow_id!r} is a batched flow but batch_variant is 'none'")
        if (c.ud, c.td) != (1, 1):
            out.append(f"Ud={c.ud}, Td={c.td}: data expansion exists only with a batch variant")
        return out
    if v not in ("spread", "folded"):
        return [f"batch_variant {v!r}: the batched launches are 'spread' (2-D grid) or 'folded' (flat grid)"]
    out = [] if _pow2(c.batch) else [f"batch must be a power of two, got {c.batch}"]
    real = effective_flow_realization(c)
    if low is not None and v not in low.batch_variants:
        out.append(f"batch_variant {v!r} has no {real!r} launch ({low.builder})")
    if v == "spread":
        if real != "matrix-resident" and not _routes(c.flow_id, frozenset({"batch-spread"})):
            out.append(f"flow {c.flow_id!r}: the spread stage cascade is flow 'batch-spread'")
        if (c.ud, c.td) != (c.batch, 1):
            out.append(f"spread launches one grid row per transform: Ud={c.batch}, Td=1 expected, "
                       f"got Ud={c.ud}, Td={c.td}")
    else:
        if low is not None and c.processing_unit not in low.folded_units:
            out.append(f"batch_variant 'folded' exists for the radix-2 stage cascade only, not "
                       f"{real}/{c.processing_unit}")
        elif c.flow_id != "batch-folded":
            out.append(f"flow {c.flow_id!r}: the folded stage cascade is flow 'batch-folded'")
        if (c.ud, c.td) != (1, c.batch):
            out.append(f"folded launches one flat grid: Ud=1, Td={c.batch} expected, got Ud={c.ud}, Td={c.td}")
    if c.fused_tile > 1 and not (real == "matrix-resident" and v == "spread"):
        out.append(f"fused_tile {c.fused_tile}: batched local groups exist only as the matrix-resident spread core")
    return out


def _rule_pipeline(c, low):
    return [] if c.pipeline == "none" else [f"pipeline {c.pipeline!r}: no such overlap schedule is built"]


RULES = (_rule_unit, _rule_layout, _rule_knobs, _rule_realization, _rule_tile, _rule_batch, _rule_pipeline)


def check_lowering(c: Candidate, profile: DeviceProfile | None = None) -> Verdict:
    """Run every rule; the candidate is legal when none objects."""
    low = LOWERINGS.get(effective_flow_realization(c))
    reasons = tuple(r for rule in RULES for r in rule(c, low))
    return Verdict(c, LoweringStatus.NOT_LOWERED if reasons else LoweringStatus.LEGAL, reasons)
