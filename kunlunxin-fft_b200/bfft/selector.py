"""Per-size runtime selector: frozen table, M0-closed, abstains out of matrix.

Same contract as the reference (src/xpu/selector.py:1-646), on the B200
table (config/selector_table.json) built from B200 measurements:

* keys (device, profile_hash, precision, transform_type, transform_direction,
  normalization, direction, N, batch); entries carrying the semantic triple
  answer only that triple, entries without it (legacy tier) answer any;
  a declared ``previous_fallbacks`` cell outranks both at its exact key;
* values (block, flow_id, flow_realization, processing_unit, params, and an
  optional measured ``executed`` runner);
* gates, in order: taxonomy, precision, profile hash (``None`` abstains), the
  table's bound env hash (absent = never selects), the caller's env hash
  (``"auto"`` recomputes it live, ``None`` abstains);
* every entry must satisfy the design space and the lowering contract or the
  whole table is refused at load time (``ConfigError``).

Host-only: no torch, no device.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

from .config import (CONFIG_DIR, NORMALIZATIONS, TRANSFORM_DIRECTIONS, TRANSFORM_TYPES,
                     ConfigError, DesignSpace, DeviceProfile)

TABLE_PATH = os.path.join(CONFIG_DIR, "selector_table.json")

# Promotion guard (percent): a challenger must beat the M0 incumbent's median
# by at least this much to enter the table (reference selector.py:63).
GUARD_PCT = 2.0

_SINGLE_RUNNERS = {
    ("global-stage", "radix2-scalar"): frozenset({"fft_dit", "fft_dif"}),
    ("global-stage", "radix4-scalar"): frozenset({"fft_dit_radix4", "fft_dif_radix4"}),
    ("matrix-resident", "dense-dot-fft64"): frozenset({"fft_dit_matrix", "fft_dif_matrix"}),
    ("fused-inplace", "radix2-scalar"): frozenset({"fft_dit_fused"}),
    ("grouped-boundary", "composite-linear-map"): frozenset({"fft_dit_grouped", "fft_dif_grouped"}),
}
_BATCH_RUNNERS = {
    ("global-stage", "radix2-scalar"): frozenset({"fft_dit_batch", "fft_dif_batch"}),
    ("global-stage", "radix4-scalar"): frozenset({"fft_dit_radix4_batch", "fft_dif_radix4_batch"}),
    ("matrix-resident", "dense-dot-fft64"): frozenset({"fft_dit_matrix_batch", "fft_dif_matrix_batch"}),
}


def _candidate_from_entry(entry: dict):
    """Schema-v2 Candidate view of one table entry (selector.py:95-137)."""
    from .candidates import LAYOUT, SPECIALIZED_ROUTING, UNIT_RADIX, Candidate

    params = dict(entry.get("params") or {})
    unit = entry.get("processing_unit")
    flow = entry.get("flow_id")
    variant = params.get("variant") or "none"
    batch = int(params.get("batch") or entry.get("batch") or 1)
    tile, rows = params.get("tile"), params.get("rows")
    local_tile = flow in (SPECIALIZED_ROUTING | {"local-fused-tile"})
    return Candidate(
        flow_id=flow, processing_unit=unit,
        radix=int(params.get("radix") or UNIT_RADIX.get(unit, 2)),
        block=int(entry.get("block") or 0),
        fused_tile=int(tile) if (local_tile and isinstance(tile, int)) else 1,
        batch=batch,
        batch_variant=variant if variant in ("spread", "folded") else "none",
        rows=int(rows) if isinstance(rows, int) else 1,
        glog=int(params.get("glog") or 0), maxp=int(params.get("maxp") or 0),
        cells=int(params.get("cells") or 1),
        flow_realization=entry.get("flow_realization") or "",
        boundary_residence=entry.get("boundary_residence") or params.get("boundary_residence") or "gm",
        pipeline=entry.get("pipeline") or params.get("pipeline") or "none",
        layout=entry.get("layout") or LAYOUT,
        ud=batch if variant == "spread" else 1,
        td=batch if variant == "folded" else 1,
    )


def entry_contract_violations(entry: dict, space: DesignSpace | None = None) -> list[str]:
    """Design-space membership + lowering-contract violations of one entry."""
    from .candidates import check_lowering

    try:
        sp = space or DesignSpace.load()
    except ConfigError as e:
        return [f"design space unreadable: {e}"]
    bad: list[str] = []
    n = entry.get("N")
    params = dict(entry.get("params") or {})
    unit = entry.get("processing_unit")
    real = entry.get("flow_realization")
    block = entry.get("block")
    if not isinstance(block, int) or block <= 0 or (block & (block - 1)):
        return [f"block {block!r} not a positive power of two"]
    tile, rows = params.get("tile"), params.get("rows")
    if unit == "radix4-scalar" and 4 not in sp.radix:
        bad.append("radix-4 not in the published radix space")
    if unit == "dense-dot-fft64":
        if tile not in sp.matrix_tiles:
            bad.append(f"tile {tile!r} not in matrix tiles {sp.matrix_tiles}")
        if rows not in sp.matrix_rows:
            bad.append(f"rows {rows!r} not in matrix rows {sp.matrix_rows}")
        if isinstance(tile, int) and isinstance(n, int) and 0 < tile <= n and n % tile:
            bad.append(f"tile {tile} does not divide N={n}")
    if unit == "radix2-scalar" and "tile" in params and real == "fused-inplace":
        if params["tile"] not in sp.fused_tile_candidates:
            bad.append(f"fused tile {params['tile']!r} not in {sp.fused_tile_candidates}")
    if unit == "composite-linear-map":
        for key, allowed in (("tile", sp.grouped_tiles), ("glog", sp.grouped_glog),
                             ("maxp", sp.grouped_maxp), ("cells", sp.grouped_cells)):
            if params.get(key) not in allowed:
                bad.append(f"{key}={params.get(key)!r} not in {allowed}")
    if "variant" in params and params["variant"] not in sp.batch_variants:
        bad.append(f"variant {params['variant']!r} not in {sp.batch_variants}")
    if "transform_type" in entry:
        tt, td, nm = (entry.get("transform_type"), entry.get("transform_direction"),
                      entry.get("normalization"))
        if tt not in TRANSFORM_TYPES:
            bad.append(f"transform_type {tt!r} not in {TRANSFORM_TYPES}")
        if td not in TRANSFORM_DIRECTIONS:
            bad.append(f"transform_direction {td!r} not in {TRANSFORM_DIRECTIONS}")
        if nm not in NORMALIZATIONS:
            bad.append(f"normalization {nm!r} not in {NORMALIZATIONS}")
    if "batch" in params and params["batch"] not in sp.batch_candidates:
        bad.append(f"batch {params['batch']!r} not in {sp.batch_candidates}")
    if "radix" in params and params["radix"] not in sp.radix:
        bad.append(f"radix {params['radix']!r} not in {sp.radix}")
    executed = entry.get("executed")
    if executed is not None:
        fam = (real, unit)
        if fam not in _SINGLE_RUNNERS:
            bad.append(f"executed {executed!r}: no known runner family for "
                       f"(flow_realization={real!r}, processing_unit={unit!r})")
        else:
            b = int(params.get("batch") or entry.get("batch") or 1)
            allowed = (_BATCH_RUNNERS if b > 1 else _SINGLE_RUNNERS).get(fam, frozenset())
            if executed not in allowed:
                bad.append(f"executed {executed!r} not a legal runner of {fam} at batch={b} "
                           f"(allowed: {sorted(allowed)})")
    if bad:
        return bad
    return list(check_lowering(_candidate_from_entry(entry)).reasons)


def semantic_key_of(entry: dict) -> tuple | None:
    if "transform_type" not in entry:
        return None
    return (entry.get("transform_type"), entry.get("transform_direction"), entry.get("normalization"))


FALLBACK_CARRY_CONTRACT = "fallback-env-binding-v1"
_FALLBACK_BINDING_KEYS = ("carry_contract", "source_env_hash", "source_profile_hash",
                          "source_precision", "source_device", "source_table_sha256",
                          "source_result_sha256", "paired_confirm")
_DEVICE_IDENTITY_KEYS = ("device_model", "multiprocessor_count", "max_shared_mem")


def fallback_binding_violations(table: dict) -> list[str]:
    """Every previous_fallbacks cell must bind to THIS table's environment,
    profile, precision and device identity (reference selector.py:279-340)."""
    out: list[str] = []
    fbs = table.get("previous_fallbacks") or ()
    if not fbs:
        return out
    ident = {k: (table.get("env") or {}).get(k) for k in _DEVICE_IDENTITY_KEYS}
    for i, e in enumerate(fbs):
        key = (e.get("N"), e.get("batch"), e.get("direction"))
        prov = e.get("previous_fallback_provenance")
        if not isinstance(prov, dict):
            out.append(f"previous_fallbacks[{i}] {key}: missing previous_fallback_provenance "
                       "(no source identity to bind against)")
            continue
        missing = [k for k in _FALLBACK_BINDING_KEYS if prov.get(k) in (None, "")]
        if missing:
            out.append(f"previous_fallbacks[{i}] {key}: provenance missing binding key(s) "
                       f"{', '.join(missing)}")
            continue
        if prov["carry_contract"] != FALLBACK_CARRY_CONTRACT:
            out.append(f"previous_fallbacks[{i}] {key}: carry_contract {prov['carry_contract']!r} "
                       f"!= {FALLBACK_CARRY_CONTRACT!r}")
        if prov["source_env_hash"] != table.get("env_hash"):
            out.append(f"previous_fallbacks[{i}] {key}: source env {prov['source_env_hash']} != table env "
                       f"{table.get('env_hash')} (stale evidence; reconfirm under the current environment)")
        if prov["source_profile_hash"] != table.get("profile_hash"):
            out.append(f"previous_fallbacks[{i}] {key}: source profile {prov['source_profile_hash']} != "
                       f"table profile {table.get('profile_hash')}")
        if prov["source_precision"] != table.get("precision"):
            out.append(f"previous_fallbacks[{i}] {key}: source precision {prov['source_precision']!r} != "
                       f"table precision {table.get('precision')!r}")
        if any(ident[k] is None for k in _DEVICE_IDENTITY_KEYS):
            out.append(f"previous_fallbacks[{i}] {key}: table carries no device identity "
                       "(env: device_model/multiprocessor_count/max_shared_mem) to bind the fallback against")
        elif prov["source_device"] != ident:
            out.append(f"previous_fallbacks[{i}] {key}: source device {prov['source_device']} != "
                       f"table device {ident}")
    return out


def is_previous_fallback(table: dict, entry: dict) -> bool:
    return any(entry is e for e in (table.get("previous_fallbacks") or ()))


def find_entry(table: dict, n: int, batch: int, direction: str, transform_type: str = "c2c",
               transform_direction: str = "forward", normalization: str = "backward") -> dict | None:
    """Previous-fallback cell first, exact semantic tier next, legacy last."""
    want = (transform_type, transform_direction, normalization)
    for e in table.get("previous_fallbacks") or ():
        if e["N"] == n and e["batch"] == batch and e["direction"] == direction \
                and semantic_key_of(e) == want:
            return e
    legacy = None
    for e in table.get("entries", ()):
        if not (e["N"] == n and e["batch"] == batch and e["direction"] == direction):
            continue
        key = semantic_key_of(e)
        if key is None:
            if legacy is None:
                legacy = e
        elif key == want:
            return e
    return legacy


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


def validate_table(table: dict, space: DesignSpace | None = None) -> list[str]:
    """All contract violations of a table dict (empty list = loadable)."""
    for key in ("profile_hash", "precision", "guard_pct", "entries"):
        if key not in table:
            return [f"selector table missing required key {key!r}"]
    violations = []
    for e in table["entries"]:
        for msg in entry_contract_violations(e, space):
            violations.append(f"entry {(e.get('N'), e.get('batch'), e.get('direction'))}: {msg}")
    seen: set = set()
    for i, e in enumerate(table.get("previous_fallbacks") or []):
        key = (e.get("N"), e.get("batch"), e.get("direction"))
        sk = semantic_key_of(e)
        if sk is None:
            violations.append(f"previous_fallbacks[{i}] {key}: missing the exact semantic triple "
                              "(transform_type/transform_direction/normalization) a per-cell fallback must claim")
        else:
            if key + sk in seen:
                violations.append(f"previous_fallbacks[{i}] {key} {sk}: duplicate previous_fallbacks cell key")
            seen.add(key + sk)
        for msg in entry_contract_violations(e, space):
            violations.append(f"previous_fallbacks[{i}] {key}: {msg}")
    return violations + fallback_binding_violations(table)


def load_table(path: str = TABLE_PATH) -> dict:
    """Load and contract-check the selector table (ConfigError on any problem)."""
    try:
        with open(path) as f:
            table = json.load(f)
    except FileNotFoundError:
        raise ConfigError(f"selector table not found: {path} (build it with "
                          "bfft.table_builder after a B200 confirmation round)") from None
    except json.JSONDecodeError as e:
        raise ConfigError(f"selector table unreadable: {path}: {e}") from None
    for key in ("profile_hash", "precision", "guard_pct", "entries"):
        if key not in table:
            raise ConfigError(f"selector table missing required key {key!r}")
    violations = validate_table(table)
    if violations:
        raise ConfigError(
            "selector table violates the shared design space / lowering contract "
            f"({len(violations)} entries): " + "; ".join(violations[:8])
            + (" ..." if len(violations) > 8 else "")
            + " -- rebuild the table from measurements under the current config/butterfly_space.json")
    return table


def assert_current_environment(table: dict) -> str:
    """Freshness gate for measurement scripts: the live env hash must equal the
    table's bound one (raises RuntimeError before any launch)."""
    bound = table.get("env_hash") or ""
    if not bound:
        raise RuntimeError("selector table carries no env_hash (pre-freshness schema); refusing to "
                           "measure against it -- rebuild the table under the current env")
    from .envcheck import current_env_hash

    cur = current_env_hash()
    if cur is None:
        raise RuntimeError("live environment fingerprint unknown (device/runtime/compiler not "
                           "probeable); cannot verify the table -- fail closed")
    if cur != bound:
        raise RuntimeError(f"environment hash {cur} != table {bound} (device/runtime/compiler changed "
                           "since the table was built); re-measure before producing new artifacts")
    return cur


def _abstain(n, direction, batch, precision, reason, tt="c2c", td="forward", nm="backward") -> Selection:
    return Selection(n=n, direction=direction, batch=batch, precision=precision, source="abstain",
                     reason=reason, transform_type=tt, transform_direction=td, normalization=nm,
                     entry_tier="abstain")


def select(direction: str, n: int, batch: int = 1, precision: str = "fp32",
           profile_hash: str | None = None, table: dict | None = None,
           env_hash: str | None = "auto", transform_type: str = "c2c",
           transform_direction: str = "forward", normalization: str = "backward") -> Selection:
    """Measured winner for one exact key, or an abstain with its reason."""
    table = table if table is not None else load_table()
    sem = (transform_type, transform_direction, normalization)
    if transform_type not in TRANSFORM_TYPES:
        return _abstain(n, direction, batch, precision,
                        f"transform_type must be one of {TRANSFORM_TYPES}, got {transform_type!r}", *sem)
    if transform_direction not in TRANSFORM_DIRECTIONS:
        return _abstain(n, direction, batch, precision,
                        f"transform_direction must be one of {TRANSFORM_DIRECTIONS}, "
                        f"got {transform_direction!r}", *sem)
    if normalization not in NORMALIZATIONS:
        return _abstain(n, direction, batch, precision,
                        f"normalization must be one of {NORMALIZATIONS}, got {normalization!r}", *sem)
    if direction not in ("dit", "dif"):
        return _abstain(n, direction, batch, precision, f"direction must be dit/dif, got {direction!r}", *sem)
    if precision != table["precision"]:
        return _abstain(n, direction, batch, precision,
                        f"table measured {table['precision']}, got {precision!r}", *sem)
    if profile_hash is None:
        return _abstain(n, direction, batch, precision,
                        "profile_hash is required; None cannot bypass the table (fall back to M0)", *sem)
    if profile_hash != table["profile_hash"]:
        return _abstain(n, direction, batch, precision,
                        f"profile hash {profile_hash} != table {table['profile_hash']}; "
                        "re-measure before selecting", *sem)
    bound = table.get("env_hash") or ""
    if not bound:
        return _abstain(n, direction, batch, precision,
                        "table carries no env_hash (pre-freshness schema); runtime selection fails "
                        "closed to M0 -- inspect entries offline via load_table only", *sem)
    cur = env_hash
    if cur == "auto":
        from .envcheck import current_env_hash

        cur = current_env_hash()
    if cur is None:
        return _abstain(n, direction, batch, precision,
                        "environment fingerprint unknown (device/runtime/compiler not probeable); "
                        "this table cannot be verified here and must fail closed to M0", *sem)
    if cur != bound:
        return _abstain(n, direction, batch, precision,
                        f"environment hash {cur} != table {bound} (device/runtime/compiler changed "
                        "since the table was built); re-run the probe and re-measure before selecting",
                        *sem)
    e = find_entry(table, n, batch, direction, *sem)
    if e is None:
        return _abstain(n, direction, batch, precision,
                        f"no measured entry for N={n} batch={batch} direction={direction} "
                        f"semantic={transform_type}/{transform_direction}/{normalization}; "
                        "fall back to M0", *sem)
    if is_previous_fallback(table, e):
        tier = "previous-fallback"
        reason = "previous-deployed per-cell fallback (issue #8): " + e.get(
            "reason", "measured confirmation winner")
    else:
        tier = "semantic" if semantic_key_of(e) is not None else "legacy"
        reason = e.get("reason", "measured confirmation winner")
    return Selection(
        n=n, direction=direction, batch=batch, precision=precision, source="table", reason=reason,
        transform_type=transform_type, transform_direction=transform_direction,
        normalization=normalization, entry_tier=tier, block=e["block"], flow_id=e["flow_id"],
        flow_realization=e["flow_realization"], processing_unit=e["processing_unit"],
        params=dict(e.get("params") or {}), incumbent_ms=e.get("incumbent_ms"),
        challenger_ms=e.get("challenger_ms"), executed=e.get("executed"))
