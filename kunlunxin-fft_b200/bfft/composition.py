"""Exact-shape composition registry (host-only).

The reference lets a 4-step decomposition (its ``run_hybrid`` flow) win
individual exact shapes through a separate, self-hashed composition table
(src/xpu/composition.py:1-240); runtime selection fails closed on any binding
or contract mismatch, and the butterfly table decides instead.  This registry
keeps that contract for the B200 library, whose 4-step core is its own
CTA-resident pass kernel (``core = "b200-pass"``), never a vendor FFT.

The contract is data: ``ENTRY_RULES`` and ``TABLE_RULES`` are ordered
(condition, message) checks over one promoted entry and over the whole
table; ``load_composition_table`` refuses a table any rule objects to, and
``composition_select`` answers only an exact (N, batch, DIT, c2c/forward/
backward) key under the table's own profile and environment.
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Callable

from .config import CONFIG_DIR, ConfigError

TABLE_PATH = os.path.join(CONFIG_DIR, "composition_table.json")
EXTERNAL_CORES_PATH = os.path.join(CONFIG_DIR, "external_cores.json")

TABLE_REQUIRED_KEYS = ("schema_version", "kind", "profile_hash", "env_hash", "precision",
                       "guard_pct", "contract_id", "entries", "source_hash", "result_sha256")
ENTRY_REQUIRED_KEYS = ("N", "batch", "direction", "precision", "tile", "core", "flow_id",
                       "flow_realization", "processing_unit", "candidate_ms", "incumbent_ms",
                       "guard_pct", "guard_pass", "reason", "evidence")
EVIDENCE_REQUIRED_KEYS = ("artifact", "artifact_sha256", "commit", "sessions", "trials",
                          "confirmation_session", "err_max", "p50_ms", "mad_ms", "p95_ms")
KIND = "composition-promotion"
CORES = ("b200-pass",)
MIN_SESSIONS = 3
MAX_ERR = 1e-4


def rows_sha256(payload) -> str:
    """sha256 of the canonical JSON of ``payload['rows']`` (or of the payload)."""
    rows = payload.get("rows", payload) if isinstance(payload, dict) else payload
    return hashlib.sha256(json.dumps(rows, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def guard_pct_of(candidate_ms: float, incumbent_ms: float) -> float:
    """Incumbent guard in percent: positive = candidate faster."""
    return (incumbent_ms - candidate_ms) / incumbent_ms * 100.0


def _missing(obj: dict, keys: tuple) -> list[str]:
    return [k for k in keys if obj.get(k) in (None, "")]


def _is_pos_int(v) -> bool:
    return isinstance(v, int) and v > 0


def _is_pow2_tile(v) -> bool:
    return isinstance(v, int) and v >= 2 and v & (v - 1) == 0


def _guard_recomputed(e) -> float:
    return guard_pct_of(float(e["candidate_ms"]), float(e["incumbent_ms"]))


Rule = tuple[Callable[..., bool], Callable[..., str]]

# (broken(entry, table), message(entry, table)); applied once the required keys are present
ENTRY_RULES: tuple[Rule, ...] = (
    (lambda e, t: e["direction"] != "dit",
     lambda e, t: f"direction {e['direction']!r} (composition flow is DIT-only)"),
    (lambda e, t: not _is_pos_int(e["N"]), lambda e, t: f"N {e['N']!r} not a positive int (exact keys only)"),
    (lambda e, t: not _is_pos_int(e["batch"]), lambda e, t: f"batch {e['batch']!r} not a positive int"),
    (lambda e, t: e.get("precision") != t.get("precision"),
     lambda e, t: f"precision {e.get('precision')!r} != table {t.get('precision')!r}"),
    (lambda e, t: e.get("core") not in CORES, lambda e, t: f"core {e.get('core')!r} not in {CORES}"),
    (lambda e, t: not _is_pow2_tile(e.get("tile")), lambda e, t: f"tile {e.get('tile')!r} invalid"),
    (lambda e, t: abs(_guard_recomputed(e) - float(e["guard_pct"])) > 1e-6,
     lambda e, t: f"guard_pct {e['guard_pct']!r} != recomputed {_guard_recomputed(e):.6f} "
                  "from candidate/incumbent ms"),
    (lambda e, t: float(e["guard_pct"]) < float(t.get("guard_pct", 2.0)),
     lambda e, t: f"guard {e['guard_pct']:.3f}% < required {t.get('guard_pct')}%"),
    (lambda e, t: e.get("guard_pass") is not True, lambda e, t: "guard_pass is not true"),
)

# (broken(evidence), message(evidence)); the evidence object of a promoted entry
EVIDENCE_RULES: tuple[Rule, ...] = (
    (lambda ev: isinstance(ev.get("err_max"), (int, float)) and float(ev["err_max"]) > MAX_ERR,
     lambda ev: f"evidence err_max {ev['err_max']} > {MAX_ERR:g} (correctness gate)"),
    (lambda ev: not ev.get("confirmation_session"),
     lambda ev: "evidence has no independent confirmation session"),
    (lambda ev: isinstance(ev.get("sessions"), int) and ev["sessions"] < MIN_SESSIONS,
     lambda ev: f"evidence sessions {ev['sessions']} < {MIN_SESSIONS}"),
)


def composition_entry_violations(entry: dict, table: dict) -> list[str]:
    """Why one promoted entry cannot be served (empty when it can)."""
    missing = _missing(entry, ENTRY_REQUIRED_KEYS)
    if missing:
        return [f"missing {k!r}" for k in missing]
    out = [msg(entry, table) for broken, msg in ENTRY_RULES if broken(entry, table)]
    ev = entry["evidence"]
    if not isinstance(ev, dict):
        return out + ["evidence not an object"]
    out += [f"evidence missing {k!r}" for k in _missing(ev, EVIDENCE_REQUIRED_KEYS)]
    return out + [msg(ev) for broken, msg in EVIDENCE_RULES if broken(ev)]


def _registered_cores(path: str) -> set:
    with open(path) as f:
        return {c.get("id") for c in json.load(f).get("cores", [])}


def table_violations(table: dict, cores_path: str = EXTERNAL_CORES_PATH) -> list[str]:
    """Why a composition table cannot be loaded (empty when it can)."""
    missing = _missing(table, TABLE_REQUIRED_KEYS)
    if missing:
        return [f"missing table key {k!r}" for k in missing]
    out = []
    if table["kind"] != KIND:
        out.append(f"kind {table['kind']!r} != {KIND!r}")
    if table.get("precision") != "fp32":
        out.append(f"precision {table.get('precision')!r} != 'fp32'")
    try:
        cores = _registered_cores(cores_path)
    except (OSError, json.JSONDecodeError) as e:
        return out + [f"core registry unreadable: {e}"]
    if table["contract_id"] not in cores:
        out.append(f"contract_id {table['contract_id']!r} not in config/external_cores.json")
    entries = table.get("entries")
    if not isinstance(entries, list) or not entries:
        return out + ["entries empty or not a list"]
    keys: list = []
    for i, e in enumerate(entries):
        if not isinstance(e, dict):
            out.append(f"entry {i} not an object")
            continue
        key = (e.get("N"), e.get("batch"), e.get("direction"))
        if key in keys:
            out.append(f"duplicate exact-shape key {key}")
        keys.append(key)
        out += [f"entry {key}: {m}" for m in composition_entry_violations(e, table)]
    if rows_sha256({"rows": entries}) != table["result_sha256"]:
        out.append("result_sha256 mismatch (entries modified after promotion)")
    return out


def load_composition_table(path: str = TABLE_PATH) -> dict | None:
    """``None`` when no table is promoted; ConfigError when one exists but is broken."""
    try:
        with open(path) as f:
            table = json.load(f)
    except FileNotFoundError:
        return None
    except json.JSONDecodeError as e:
        raise ConfigError(f"composition table unreadable: {path}: {e}") from None
    if not isinstance(table, dict):
        raise ConfigError(f"composition table is not an object: {path}")
    problems = table_violations(table)
    if problems:
        raise ConfigError(f"composition table violates its contract ({len(problems)}): "
                          + "; ".join(problems[:8]) + (" ..." if len(problems) > 8 else "")
                          + " -- re-promote from the confirmation evidence")
    return table


def _binds(table: dict, precision: str, profile_hash: str | None, env_hash: str | None) -> bool:
    """The caller's precision, profile and environment are the table's."""
    if precision != table.get("precision") or not profile_hash or profile_hash != table.get("profile_hash"):
        return False
    bound = table.get("env_hash") or ""
    if not bound:
        return False
    if env_hash == "auto":
        from .envcheck import current_env_hash

        env_hash = current_env_hash()
    return env_hash is not None and env_hash == bound


def composition_select(direction: str, n: int, batch: int = 1, precision: str = "fp32",
                       profile_hash: str | None = None, env_hash: str | None = "auto",
                       table: dict | None = None, transform_type: str = "c2c",
                       transform_direction: str = "forward",
                       normalization: str = "backward") -> dict | None:
    """The promoted entry for this exact key, or ``None`` (fail closed)."""
    if direction != "dit" or (transform_type, transform_direction, normalization) != ("c2c", "forward", "backward"):
        return None
    table = table if table is not None else load_composition_table()
    if table is None or not _binds(table, precision, profile_hash, env_hash):
        return None
    return next((e for e in table["entries"] if (e["N"], e["batch"], e["direction"]) == (n, batch, direction)),
                None)
