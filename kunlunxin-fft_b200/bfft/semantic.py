"""Per-semantic candidate families and legality (host-only).

Same membership rules as the reference (src/xpu/semantic.py:33-125): every
semantic reaches the shared butterfly cores through its own wrapper, and the
dedicated real-transform flows belong only to their own transform type.
"""
from __future__ import annotations

from dataclasses import dataclass

from .config import NORMALIZATIONS, TRANSFORM_DIRECTIONS, TRANSFORM_TYPES

SEMANTIC_SPECS: dict[str, tuple[str, str, str]] = {
    "c2c-forward": ("c2c", "forward", "backward"),
    "c2c-inverse": ("c2c", "inverse", "backward"),
    "r2c": ("r2c", "forward", "backward"),
    "c2r": ("c2r", "inverse", "backward"),
}

CORE_FLOWS = frozenset({"baseline-global-stage", "batch-spread", "batch-folded", "local-fused-tile"})

SPECIALIZED_FLOWS: dict[str, frozenset] = {
    "c2c": frozenset(),
    "r2c": frozenset({"dedicated-r2c-pack-v1"}),
    "c2r": frozenset({"dedicated-c2r-hermitian-v1"}),
}


@dataclass(frozen=True)
class SemanticSpec:
    label: str
    transform_type: str
    transform_direction: str
    normalization: str

    @property
    def key(self) -> tuple:
        return (self.transform_type, self.transform_direction, self.normalization)


def spec(label: str) -> SemanticSpec:
    if label not in SEMANTIC_SPECS:
        raise KeyError(f"unknown semantic label {label!r}; known: {sorted(SEMANTIC_SPECS)}")
    return SemanticSpec(label, *SEMANTIC_SPECS[label])


def family(transform_type: str) -> frozenset:
    """Legal flow ids for one transform type (core + specialized)."""
    if transform_type not in TRANSFORM_TYPES:
        raise KeyError(f"unknown transform_type {transform_type!r}; known: {TRANSFORM_TYPES}")
    return CORE_FLOWS | SPECIALIZED_FLOWS[transform_type]


def family_allows(transform_type: str, flow_id: str) -> bool:
    return flow_id in family(transform_type)


def family_size(transform_type: str) -> int:
    return len(family(transform_type))


def validate_taxonomy() -> list[str]:
    bad = []
    for label, (tt, tdir, norm) in SEMANTIC_SPECS.items():
        if tt not in TRANSFORM_TYPES:
            bad.append(f"{label}: transform_type {tt!r} not in taxonomy")
        if tdir not in TRANSFORM_DIRECTIONS:
            bad.append(f"{label}: transform_direction {tdir!r} not in taxonomy")
        if norm not in NORMALIZATIONS:
            bad.append(f"{label}: normalization {norm!r} not in taxonomy")
    for tt in TRANSFORM_TYPES:
        if tt not in SPECIALIZED_FLOWS:
            bad.append(f"SPECIALIZED_FLOWS missing {tt!r}")
    return bad
