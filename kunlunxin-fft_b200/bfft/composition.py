"""Exact-shape composition registry (host-only).

The reference promotes a 4-step decomposition (its ``run_hybrid`` flow) for
individual exact shapes through a separate, self-hashed composition table
(src/xpu/composition.py:1-240); runtime selection fails closed on any
binding or contract mismatch so the butterfly table decides instead.  The
B200 registry keeps that contract.  Its core is this library's own
CTA-resident pass kernel (``core = "b200-pass"``), never a vendor FFT.
"""
from __future__ import annotations

import hashlib
import json
import os

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


def rows_sha256(payload) -> str:
    """sha256 of the canonical JSON of ``payload['rows']`` (or the payload)."""
    rows = payload.get("rows", payload) if isinstance(payload, dict) else payload
    return hashlib.sha256(json.dumps(rows, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def guard_pct_of(candidate_ms: float, incumbent_ms: float) -> float:
    """Incumbent guard in percent: positive = candidate faster."""
    return (incumbent_ms - candidate_ms) / incumbent_ms * 100.0


def composition_entry_violations(entry: dict, table: dict) -> list[str]:
    bad = [f"missing {k!r}" for k in ENTRY_REQUIRED_KEYS if entry.get(k) in (None, "")]
    if bad:
        return bad
    if entry["direction"] != "dit":
        bad.append(f"direction {entry['direction']!r} (composition flow is DIT-only)")
    if not isinstance(entry["N"], int) or entry["N"] <= 0:
        bad.append(f"N {entry['N']!r} not a positive int (exact keys only)")
    if not isinstance(entry["batch"], int) or entry["batch"] <= 0:
        bad.append(f"batch {entry['batch']!r} not a positive int")
    if entry.get("precision") != table.get("precision"):
        bad.append(f"precision {entry.get('precision')!r} != table {table.get('precision')!r}")
    if entry.get("core") not in CORES:
        bad.append(f"core {entry.get('core')!r} not in {CORES}")
    tile = entry.get("tile")
    if not isinstance(tile, int) or tile < 2 or tile & (tile - 1):
        bad.append(f"tile {tile!r} invalid")
    recomputed = guard_pct_of(float(entry["candidate_ms"]), float(entry["incumbent_ms"]))
    if abs(recomputed - float(entry["guard_pct"])) > 1e-6:
        bad.append(f"guard_pct {entry['guard_pct']!r} != recomputed {recomputed:.6f} from candidate/incumbent ms")
    if float(entry["guard_pct"]) < float(table.get("guard_pct", 2.0)):
        bad.append(f"guard {entry['guard_pct']:.3f}% < required {table.get('guard_pct')}%")
    if entry.get("guard_pass") is not True:
        bad.append("guard_pass is not true")
    ev = entry.get("evidence")
    if not isinstance(ev, dict):
        return bad + ["evidence not an object"]
    bad += [f"evidence missing {k!r}" for k in EVIDENCE_REQUIRED_KEYS if ev.get(k) in (None, "")]
    if isinstance(ev.get("err_max"), (int, float)) and float(ev["err_max"]) > 1e-4:
        bad.append(f"evidence err_max {ev['err_max']} > 1e-4 (correctness gate)")
    if not ev.get("confirmation_session"):
        bad.append("evidence has no independent confirmation session")
    if isinstance(ev.get("sessions"), int) and ev["sessions"] < 3:
        bad.append(f"evidence sessions {ev['sessions']} < 3")
    return bad


def table_violations(table: dict, cores_path: str = EXTERNAL_CORES_PATH) -> list[str]:
    bad = [f"missing table key {k!r}" for k in TABLE_REQUIRED_KEYS if table.get(k) in (None, "")]
    if bad:
        return bad
    if table["kind"] != KIND:
        bad.append(f"kind {table['kind']!r} != {KIND!r}")
    if table.get("precision") != "fp32":
        bad.append(f"precision {table.get('precision')!r} != 'fp32'")
    try:
        with open(cores_path) as f:
            ids = {c.get("id") for c in json.load(f).get("cores", [])}
    except (OSError, json.JSONDecodeError) as e:
        return bad + [f"core registry unreadable: {e}"]
    if table["contract_id"] not in ids:
        bad.append(f"contract_id {table['contract_id']!r} not in config/external_cores.json")
    entries = table.get("entries")
    if not isinstance(entries, list) or not entries:
        bad.append("entries empty or not a list")
        entries = []
    seen: set = set()
    for i, e in enumerate(entries):
        if not isinstance(e, dict):
            bad.append(f"entry {i} not an object")
            continue
        key = (e.get("N"), e.get("batch"), e.get("direction"))
        if key in seen:
            bad.append(f"duplicate exact-shape key {key}")
        seen.add(key)
        bad.extend(f"entry {key}: {m}" for m in composition_entry_violations(e, table))
    if entries and rows_sha256({"rows": entries}) != table["result_sha256"]:
        bad.append("result_sha256 mismatch (entries modified after promotion)")
    return bad


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
    v = table_violations(table)
    if v:
        raise ConfigError(f"composition table violates its contract ({len(v)}): " + "; ".join(v[:8])
                          + (" ..." if len(v) > 8 else "")
                          + " -- re-promote from the confirmation evidence")
    return table


def composition_select(direction: str, n: int, batch: int = 1, precision: str = "fp32",
                       profile_hash: str | None = None, env_hash: str | None = "auto",
                       table: dict | None = None, transform_type: str = "c2c",
                       transform_direction: str = "forward",
                       normalization: str = "backward") -> dict | None:
    """Exact-shape composition entry, or ``None`` (fail closed)."""
    if direction != "dit":
        return None
    if (transform_type, transform_direction, normalization) != ("c2c", "forward", "backward"):
        return None
    if table is None:
        table = load_composition_table()
        if table is None:
            return None
    if precision != table.get("precision"):
        return None
    if not profile_hash or profile_hash != table.get("profile_hash"):
        return None
    bound = table.get("env_hash") or ""
    if not bound:
        return None
    if env_hash == "auto":
        from .envcheck import current_env_hash

        env_hash = current_env_hash()
    if env_hash is None or env_hash != bound:
        return None
    for e in table["entries"]:
        if e["N"] == n and e["batch"] == batch and e["direction"] == direction:
            return e
    return None
