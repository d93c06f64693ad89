"""Runtime selector over the frozen B200 table (host-only: no torch, no device).

Behaviour follows the reference's selector (src/xpu/selector.py:1-646): one
measured winner per exact key, M0 when the table cannot answer, and a table
that breaks the design space or the lowering contract is refused whole at
load time (``ConfigError``).  The data is the B200 table
(config/selector_table.json) that ``bfft.table_builder`` builds from B200
measurements.

The module is organised around three declarative pieces:

* ``GATES`` -- the ordered checks a query must pass before the table is
  consulted (taxonomy, direction, precision, profile hash, the table's bound
  environment hash, the caller's environment hash); the first failing gate's
  reason is the abstain reason;
* ``_TIERS`` -- where an answer may come from, highest priority first: a
  declared previous-fallback cell at its exact key, an entry of the exact
  semantic triple, an entry without a triple (legacy tier);
* ``ENTRY_RULES`` / ``PROVENANCE_RULES`` -- the contract every entry and
  every previous-fallback cell must meet, as (condition, message) rules.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from functools import cached_property
from typing import Callable

from .config import (CONFIG_DIR, NORMALIZATIONS, TRANSFORM_DIRECTIONS, TRANSFORM_TYPES,
                     ConfigError, DesignSpace, DeviceProfile)

TABLE_PATH = os.path.join(CONFIG_DIR, "selector_table.json")

# Promotion guard (percent): a challenger enters the table only when it beats
# the M0 incumbent's median by at least this much (reference selector.py:63).
GUARD_PCT = 2.0

REQUIRED_TABLE_KEYS = ("profile_hash", "precision", "guard_pct", "entries")
FALLBACK_CARRY_CONTRACT = "fallback-env-binding-v1"
DEVICE_IDENTITY_KEYS = ("device_model", "multiprocessor_count", "max_shared_mem")

# Runner functions per (flow_realization, processing_unit): single transform, batched.
RUNNER_FAMILIES = {
    ("global-stage", "radix2-scalar"): (("fft_dit", "fft_dif"), ("fft_dit_batch", "fft_dif_batch")),
    ("global-stage", "radix4-scalar"): (("fft_dit_radix4", "fft_dif_radix4"),
                                        ("fft_dit_radix4_batch", "fft_dif_radix4_batch")),
    ("matrix-resident", "dense-dot-fft64"): (("fft_dit_matrix", "fft_dif_matrix"),
                                             ("fft_dit_matrix_batch", "fft_dif_matrix_batch")),
    ("fused-inplace", "radix2-scalar"): (("fft_dit_fused",), ()),
    ("grouped-boundary", "composite-linear-map"): (("fft_dit_grouped", "fft_dif_grouped"), ()),
}


def semantic_key_of(entry: dict) -> tuple | None:
    """(transform_type, transform_direction, normalization) of an entry, None for the legacy tier."""
    if "transform_type" not in entry:
        return None
    return (entry.get("transform_type"), entry.get("transform_direction"), entry.get("normalization"))


def _shape(entry: dict) -> tuple:
    return (entry.get("N"), entry.get("batch"), entry.get("direction"))


# ================================================================ entry contract

def _candidate_of(entry: dict):
    """The Candidate (lowering-contract view) an entry describes."""
    from .candidates import LAYOUT, SPECIALIZED_ROUTING, UNIT_RADIX, Candidate

    p = dict(entry.get("params") or {})
    flow, unit = entry.get("flow_id"), entry.get("processing_unit")
    variant = p.get("variant") if p.get("variant") in ("spread", "folded") else "none"
    batch = int(p.get("batch") or entry.get("batch") or 1)
    has_local_group = flow == "local-fused-tile" or flow in SPECIALIZED_ROUTING
    tile, rows = p.get("tile"), p.get("rows")
    return Candidate(
        flow_id=flow, processing_unit=unit, radix=int(p.get("radix") or UNIT_RADIX.get(unit, 2)),
        block=int(entry.get("block") or 0),
        fused_tile=tile if has_local_group and isinstance(tile, int) else 1,
        batch=batch, batch_variant=variant, rows=rows if isinstance(rows, int) else 1,
        glog=int(p.get("glog") or 0), maxp=int(p.get("maxp") or 0), cells=int(p.get("cells") or 1),
        flow_realization=entry.get("flow_realization") or "",
        boundary_residence=entry.get("boundary_residence") or p.get("boundary_residence") or "gm",
        pipeline=entry.get("pipeline") or p.get("pipeline") or "none",
        layout=entry.get("layout") or LAYOUT,
        ud=batch if variant == "spread" else 1, td=batch if variant == "folded" else 1)


def _knob_domains(entry: dict, sp: DesignSpace) -> list[tuple[str, object, object]]:
    """(knob, value, allowed values) for every knob the entry's unit consumes."""
    p = dict(entry.get("params") or {})
    unit, real = entry.get("processing_unit"), entry.get("flow_realization")
    out = []
    if unit == "dense-dot-fft64":
        out += [("tile", p.get("tile"), sp.matrix_tiles), ("rows", p.get("rows"), sp.matrix_rows)]
    if unit == "radix2-scalar" and real == "fused-inplace" and "tile" in p:
        out.append(("fused tile", p["tile"], sp.fused_tile_candidates))
    if unit == "composite-linear-map":
        out += [("tile", p.get("tile"), sp.grouped_tiles), ("glog", p.get("glog"), sp.grouped_glog),
                ("maxp", p.get("maxp"), sp.grouped_maxp), ("cells", p.get("cells"), sp.grouped_cells)]
    for key, allowed in (("variant", sp.batch_variants), ("batch", sp.batch_candidates), ("radix", sp.radix)):
        if key in p:
            out.append((key, p[key], allowed))
    return out


def _rule_knobs(entry, sp):
    msgs = [f"{name}={val!r} is outside the design space {allowed}"
            for name, val, allowed in _knob_domains(entry, sp) if val not in allowed]
    if entry.get("processing_unit") == "radix4-scalar" and 4 not in sp.radix:
        msgs.append("radix-4 is not in the published radix space")
    tile, n = (entry.get("params") or {}).get("tile"), entry.get("N")
    if entry.get("processing_unit") == "dense-dot-fft64" and isinstance(tile, int) and isinstance(n, int) \
            and 0 < tile <= n and n % tile:
        msgs.append(f"tile {tile} does not divide N={n}")
    return msgs


def _rule_semantics(entry, sp):
    if "transform_type" not in entry:
        return []
    return [f"{key} {entry.get(key)!r} is not one of {allowed}"
            for key, allowed in (("transform_type", TRANSFORM_TYPES), ("transform_direction", TRANSFORM_DIRECTIONS),
                                 ("normalization", NORMALIZATIONS)) if entry.get(key) not in allowed]


def _rule_executed(entry, sp):
    executed = entry.get("executed")
    if executed is None:
        return []
    fam = (entry.get("flow_realization"), entry.get("processing_unit"))
    if fam not in RUNNER_FAMILIES:
        return [f"executed {executed!r}: (flow_realization, processing_unit) = {fam} names no runner family"]
    batch = int((entry.get("params") or {}).get("batch") or entry.get("batch") or 1)
    allowed = RUNNER_FAMILIES[fam][1 if batch > 1 else 0]
    if executed not in allowed:
        return [f"executed {executed!r} does not run {fam} at batch={batch} (its runners: {sorted(allowed)})"]
    return []


ENTRY_RULES: tuple[Callable[[dict, DesignSpace], list[str]], ...] = (_rule_knobs, _rule_semantics, _rule_executed)


def entry_contract_violations(entry: dict, space: DesignSpace | None = None) -> list[str]:
    """Why an entry cannot be served (design space, runner family, lowering
    contract); empty when it can."""
    from .candidates import check_lowering

    try:
        sp = space or DesignSpace.load()
    except ConfigError as e:
        return [f"design space unreadable: {e}"]
    block = entry.get("block")
    if not isinstance(block, int) or block <= 0 or block & (block - 1):
        return [f"block {block!r} is not a positive power of two"]
    msgs = [m for rule in ENTRY_RULES for m in rule(entry, sp)]
    return msgs or list(check_lowering(_candidate_of(entry)).reasons)


# ================================================================ previous-fallback cells

def _device_identity(table: dict) -> dict:
    env = table.get("env") or {}
    return {k: env.get(k) for k in DEVICE_IDENTITY_KEYS}


# (provenance key, what the table says it must be, message for a mismatch)
PROVENANCE_RULES = (
    ("carry_contract", lambda t: FALLBACK_CARRY_CONTRACT, "carry_contract {got!r} != {want!r}"),
    ("source_env_hash", lambda t: t.get("env_hash"),
     "source env {got} != table env {want} (stale evidence; reconfirm under the current environment)"),
    ("source_profile_hash", lambda t: t.get("profile_hash"), "source profile {got} != table profile {want}"),
    ("source_precision", lambda t: t.get("precision"), "source precision {got!r} != table precision {want!r}"),
)
PROVENANCE_KEYS = ("carry_contract", "source_env_hash", "source_profile_hash", "source_precision",
                   "source_device", "source_table_sha256", "source_result_sha256", "paired_confirm")


def _cell_binding_problems(cell: dict, table: dict) -> list[str]:
    prov = cell.get("previous_fallback_provenance")
    if not isinstance(prov, dict):
        return ["missing previous_fallback_provenance (no source identity to bind against)"]
    missing = [k for k in PROVENANCE_KEYS if prov.get(k) in (None, "")]
    if missing:
        return ["provenance missing binding key(s) " + ", ".join(missing)]
    msgs = [msg.format(got=prov[key], want=want(table))
            for key, want, msg in PROVENANCE_RULES if prov[key] != want(table)]
    ident = _device_identity(table)
    if any(v is None for v in ident.values()):
        msgs.append("table carries no device identity (env: device_model/multiprocessor_count/max_shared_mem) "
                    "to bind the fallback against")
    elif prov["source_device"] != ident:
        msgs.append(f"source device {prov['source_device']} != table device {ident}")
    return msgs


def fallback_binding_violations(table: dict) -> list[str]:
    """Every previous_fallbacks cell binds to THIS table's environment,
    profile, precision and device identity (reference selector.py:279-340)."""
    return [f"previous_fallbacks[{i}] {_shape(cell)}: {m}"
            for i, cell in enumerate(table.get("previous_fallbacks") or ())
            for m in _cell_binding_problems(cell, table)]


def is_previous_fallback(table: dict, entry: dict) -> bool:
    return any(entry is cell for cell in (table.get("previous_fallbacks") or ()))


# ================================================================ table lookup

@dataclass(frozen=True)
class _Index:
    """Where each exact key can be answered from, per tier."""

    fallback: dict
    semantic: dict
    legacy: dict

    @classmethod
    def of(cls, table: dict) -> "_Index":
        fb: dict = {}
        for cell in table.get("previous_fallbacks") or ():
            fb.setdefault((*_shape(cell), semantic_key_of(cell)), cell)
        sem: dict = {}
        leg: dict = {}
        for e in table.get("entries", ()):
            k = semantic_key_of(e)
            if k is None:
                leg.setdefault(_shape(e), e)
            else:
                sem.setdefault((*_shape(e), k), e)
        return cls(fb, sem, leg)


# highest priority first: (tier name, lookup)
_TIERS = (
    ("previous-fallback", lambda ix, shape, sem: ix.fallback.get((*shape, sem))),
    ("semantic", lambda ix, shape, sem: ix.semantic.get((*shape, sem))),
    ("legacy", lambda ix, shape, sem: ix.legacy.get(shape)),
)


def _lookup(table: dict, n: int, batch: int, direction: str, sem: tuple) -> tuple[str | None, dict | None]:
    ix = _Index.of(table)
    for tier, get in _TIERS:
        e = get(ix, (n, batch, direction), sem)
        if e is not None:
            return tier, e
    return None, None


def find_entry(table: dict, n: int, batch: int, direction: str, transform_type: str = "c2c",
               transform_direction: str = "forward", normalization: str = "backward") -> dict | None:
    """The entry answering one exact key (previous-fallback cell, then the
    exact semantic tier, then the legacy tier), or None."""
    return _lookup(table, n, batch, direction, (transform_type, transform_direction, normalization))[1]


@dataclass(frozen=True)
class Selection:
    """One selector verdict; ``source`` is ``table`` or ``abstain``."""

    n: int
    direction: str
    batch: int
    precision: str
    source: str
    reason: str
    transform_type: str = "c2c"
    transform_direction: str = "forward"
    normalization: str = "backward"
    entry_tier: str = "abstain"
    block: int | None = None
    flow_id: str | None = None
    flow_realization: str | None = None
    processing_unit: str | None = None
    params: dict = field(default_factory=dict)
    incumbent_ms: float | None = None
    challenger_ms: float | None = None
    executed: str | None = None

    @property
    def selected(self) -> bool:
        return self.source == "table"


# ================================================================ loading

def validate_table(table: dict, space: DesignSpace | None = None) -> list[str]:
    """All contract violations of a table dict (empty list = loadable)."""
    missing = [k for k in REQUIRED_TABLE_KEYS if k not in table]
    if missing:
        return [f"selector table missing required key {missing[0]!r}"]
    out = [f"entry {_shape(e)}: {m}" for e in table["entries"] for m in entry_contract_violations(e, space)]
    seen: set = set()
    for i, cell in enumerate(table.get("previous_fallbacks") or ()):
        sk = semantic_key_of(cell)
        if sk is None:
            out.append(f"previous_fallbacks[{i}] {_shape(cell)}: missing the exact semantic triple "
                       "(transform_type/transform_direction/normalization) a per-cell fallback must claim")
        elif (*_shape(cell), sk) in seen:
            out.append(f"previous_fallbacks[{i}] {_shape(cell)} {sk}: duplicate previous_fallbacks cell key")
        else:
            seen.add((*_shape(cell), sk))
        out += [f"previous_fallbacks[{i}] {_shape(cell)}: {m}" for m in entry_contract_violations(cell, space)]
    return out + fallback_binding_violations(table)


def load_table(path: str = TABLE_PATH) -> dict:
    """Read and contract-check the selector table (ConfigError on any problem)."""
    try:
        with open(path) as f:
            table = json.load(f)
    except FileNotFoundError:
        raise ConfigError(f"selector table not found: {path} (build it with "
                          "bfft.table_builder after a B200 confirmation round)") from None
    except json.JSONDecodeError as e:
        raise ConfigError(f"selector table unreadable: {path}: {e}") from None
    problems = validate_table(table)
    if problems and problems[0].startswith("selector table missing required key"):
        raise ConfigError(problems[0])
    if problems:
        shown = "; ".join(problems[:8]) + (" ..." if len(problems) > 8 else "")
        raise ConfigError(f"selector table violates the shared design space / lowering contract "
                          f"({len(problems)} entries): {shown} -- rebuild the table from measurements under "
                          "the current config/butterfly_space.json")
    return table


def assert_current_environment(table: dict) -> str:
    """Freshness gate for measurement scripts: the live environment hash must
    equal the table's bound one (RuntimeError otherwise, before any launch)."""
    from .envcheck import current_env_hash

    bound = table.get("env_hash") or ""
    if not bound:
        raise RuntimeError("selector table carries no env_hash (pre-freshness schema); refusing to "
                           "measure against it -- rebuild the table under the current env")
    cur = current_env_hash()
    if cur is None:
        raise RuntimeError("live environment fingerprint unknown (device/runtime/compiler not "
                           "probeable); cannot verify the table -- fail closed")
    if cur != bound:
        raise RuntimeError(f"environment hash {cur} != table {bound} (device/runtime/compiler changed "
                           "since the table was built); re-measure before producing new artifacts")
    return cur


# ================================================================ selection

@dataclass(frozen=True)
class _Query:
    direction: str
    n: int
    batch: int
    precision: str
    profile_hash: str | None
    env_hash: str | None
    sem: tuple
    table: dict = field(repr=False, compare=False)

    @cached_property
    def live_env(self) -> str | None:
        """The caller's environment hash ("auto" = fingerprint this process now)."""
        if self.env_hash != "auto":
            return self.env_hash
        from .envcheck import current_env_hash

        return current_env_hash()


# (fails, reason) in the order the reference applies them (selector.py:524-608)
GATES: tuple[tuple[Callable[[_Query], bool], Callable[[_Query], str]], ...] = (
    (lambda q: q.sem[0] not in TRANSFORM_TYPES,
     lambda q: f"transform_type must be one of {TRANSFORM_TYPES}, got {q.sem[0]!r}"),
    (lambda q: q.sem[1] not in TRANSFORM_DIRECTIONS,
     lambda q: f"transform_direction must be one of {TRANSFORM_DIRECTIONS}, got {q.sem[1]!r}"),
    (lambda q: q.sem[2] not in NORMALIZATIONS,
     lambda q: f"normalization must be one of {NORMALIZATIONS}, got {q.sem[2]!r}"),
    (lambda q: q.direction not in ("dit", "dif"),
     lambda q: f"direction must be dit/dif, got {q.direction!r}"),
    (lambda q: q.precision != q.table["precision"],
     lambda q: f"table measured {q.table['precision']}, got {q.precision!r}"),
    (lambda q: q.profile_hash is None,
     lambda q: "profile_hash is required; None cannot bypass the table (fall back to M0)"),
    (lambda q: q.profile_hash != q.table["profile_hash"],
     lambda q: f"profile hash {q.profile_hash} != table {q.table['profile_hash']}; re-measure before selecting"),
    (lambda q: not (q.table.get("env_hash") or ""),
     lambda q: "table carries no env_hash (pre-freshness schema); runtime selection fails closed to M0 -- "
               "inspect entries offline via load_table only"),
    (lambda q: q.live_env is None,
     lambda q: "environment fingerprint unknown (device/runtime/compiler not probeable); this table cannot "
               "be verified here and must fail closed to M0"),
    (lambda q: q.live_env != q.table.get("env_hash"),
     lambda q: f"environment hash {q.live_env} != table {q.table.get('env_hash')} (device/runtime/compiler "
               "changed since the table was built); re-run the probe and re-measure before selecting"),
)


def select(direction: str, n: int, batch: int = 1, precision: str = "fp32",
           profile_hash: str | None = None, table: dict | None = None,
           env_hash: str | None = "auto", transform_type: str = "c2c",
           transform_direction: str = "forward", normalization: str = "backward") -> Selection:
    """The measured winner for one exact key, or an abstain with its reason."""
    table = table if table is not None else load_table()
    q = _Query(direction, n, batch, precision, profile_hash, env_hash,
               (transform_type, transform_direction, normalization), table)
    common = dict(n=n, direction=direction, batch=batch, precision=precision, transform_type=transform_type,
                  transform_direction=transform_direction, normalization=normalization)
    for fails, reason in GATES:
        if fails(q):
            return Selection(source="abstain", reason=reason(q), entry_tier="abstain", **common)
    tier, e = _lookup(table, n, batch, direction, q.sem)
    if e is None:
        return Selection(source="abstain", entry_tier="abstain", **common,
                         reason=f"no measured entry for N={n} batch={batch} direction={direction} "
                                f"semantic={transform_type}/{transform_direction}/{normalization}; fall back to M0")
    reason = e.get("reason", "measured confirmation winner")
    if tier == "previous-fallback":
        reason = "previous-deployed per-cell fallback (issue #8): " + reason
    return Selection(source="table", reason=reason, entry_tier=tier, block=e["block"], flow_id=e["flow_id"],
                     flow_realization=e["flow_realization"], processing_unit=e["processing_unit"],
                     params=dict(e.get("params") or {}), incumbent_ms=e.get("incumbent_ms"),
                     challenger_ms=e.get("challenger_ms"), executed=e.get("executed"), **common)
