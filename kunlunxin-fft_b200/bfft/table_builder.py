"""Selector table builder and the B200 re-profiling workflow.

The frozen selector table (``config/selector_table.json``) is the only thing
``plan_fft`` consults, so it is rebuilt from B200 measurements whenever the
device, driver, CUDA stack or library changes (the table binds the
environment hash it was measured under and the selector abstains to M0 on any
other).  Two stages, after the reference's workflow
(``scripts/build_selector_table.py``, ``src/xpu/evidence.py:25-67``,
``scripts/hw_probe.py``):

``measure`` (on a B200)
    For every shape of the size matrix, every candidate lowering the design
    space allows is timed in interleaved sessions (the candidate order is
    reshuffled every session), ``trials`` executions per session, each one
    bracketed by CUDA events with the device kept busy ahead of it so that
    host launch overhead is not counted.  Each candidate's maximum relative
    L2 error per transform against float64 ``numpy.fft`` (sampled rows) is
    recorded beside its timings.  The run file carries its manifest: device,
    profile and environment hashes, precision, protocol and the correctness
    threshold.

``build`` (anywhere)
    Runs whose manifests disagree are refused.  A candidate may enter a
    comparison only with complete evidence (:func:`candidate_verdict`): present
    in every session, every trial timed, finite positive median, error below
    the threshold.  Per shape the incumbent is M0 (B = 1) or the faster M4
    variant (B > 1); the fastest admissible challenger becomes the entry when
    its median (median of session medians) beats the incumbent's by at least
    ``GUARD_PCT`` percent.  Batched shapes whose challengers all miss the guard
    keep the faster M4 variant as their entry.  The written table passes
    ``selector.validate_table`` or nothing is written.

    python -m bfft.table_builder measure --out run.json [--quick]
    python -m bfft.table_builder build run.json [...] --out config/selector_table.json
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import random
import statistics
import sys
import time
from dataclasses import dataclass

from .config import ConfigError, DesignSpace, DeviceProfile
from .selector import GUARD_PCT, TABLE_PATH, validate_table

PROTOCOL_ID = "b200-interleaved-sessions-v1"
TIMING_SCOPE = "device: CUDA events around one execute_fft_plan call, device kept busy ahead of the start event"
SELECTION_SEMANTICS = ("median of per-session medians (interleaved sessions within one run), challenger vs "
                       "incumbent under the promotion guard; not paired per-trial medians")
MANIFEST_KEYS = ("device", "profile_hash", "env_hash", "precision", "dtype", "correctness_threshold", "warmup",
                 "trials", "sessions", "timing_scope", "protocol_id")
DEFAULT_THRESHOLD = 1e-6
REAL_FLOWS = {"r2c": "dedicated-r2c-pack-v1", "c2r": "dedicated-c2r-hermitian-v1"}


# ---------------------------------------------------------------- shapes and candidates

@dataclass(frozen=True)
class Shape:
    n: int
    batch: int
    direction: str
    transform_type: str = "c2c"
    transform_direction: str = "forward"
    normalization: str = "backward"
    semantic: bool = False  # entry carries the (type, direction, norm) triple

    @property
    def key(self) -> str:
        return (f"N{self.n}B{self.batch}:{self.direction}:{self.transform_type}-{self.transform_direction}-"
                f"{self.normalization}{':sem' if self.semantic else ''}")

    def as_dict(self) -> dict:
        return {"n": self.n, "batch": self.batch, "direction": self.direction,
                "transform_type": self.transform_type, "transform_direction": self.transform_direction,
                "normalization": self.normalization, "semantic": self.semantic}


def default_shapes(quick: bool = False) -> list[Shape]:
    """The size matrix of the B200 table: the BASELINE configurations.

    Legacy (any-semantic) tier: c2c forward at B = 1 for N = 2^4..2^20 in
    both directions, the batched configurations 2 and 3 (B * N = 2^24) and
    5a.  Semantic tier: the inverse of configuration 2 and the real
    transforms of configuration 4."""
    if quick:
        return [Shape(1024, 1, "dit"), Shape(4096, 4096, "dit"),
                Shape(4096, 256, "dit", "r2c", "forward", "backward", True)]
    out: list[Shape] = []
    for l in range(4, 21):
        for d in ("dit", "dif"):
            out.append(Shape(1 << l, 1, d))
    batched = {(1024, 16), (1024, 64), (2048, 16), (2048, 64), (65536, 8192)}
    batched |= {(1 << l, 1 << (24 - l)) for l in range(4, 21)}
    for n, b in sorted(batched):
        out.append(Shape(n, b, "dit"))
    for n, b in ((1024, 16), (1024, 64), (2048, 16), (2048, 64)):
        out.append(Shape(n, b, "dit", "c2c", "inverse", "backward", True))
    for n in (4096, 16384, 65536):
        out.append(Shape(n, 256, "dit", "r2c", "forward", "backward", True))
        out.append(Shape(n, 256, "dit", "c2r", "inverse", "backward", True))
    return out


def _desc(flow, real, unit, params, block=256, executed=None) -> dict:
    d = {"block": block, "flow_id": flow, "flow_realization": real, "processing_unit": unit, "params": params}
    if executed:
        d["executed"] = executed
    return d


def candidates(shape: Shape, space: DesignSpace | None = None) -> tuple[dict, list[str]]:
    """({candidate key: descriptor}, incumbent keys) of one shape.

    A descriptor is the schema-v2 attribution of a table entry (block,
    flow_id, flow_realization, processing_unit, params[, executed]); the key
    names the lowering like the reference's bench keys (m0 / m1 / m2 / m3 /
    m4 / m5)."""
    sp = space or DesignSpace.load()
    n, b, d = shape.n, shape.batch, shape.direction
    l = n.bit_length() - 1
    cands: dict[str, dict] = {}
    if shape.transform_type in REAL_FLOWS:
        # The incumbent is the packed compat flow on M4 folded (the M0
        # fallback of a batched real transform); challengers are the
        # dedicated half-length flows on the batch local-fused core.
        cands[f"m4_folded_{d}"] = _desc("batch-folded", "global-stage", "radix2-scalar",
                                        {"variant": "folded", "batch": b})
        flow = REAL_FLOWS[shape.transform_type]
        half = n // 2
        for core_dir in ("dit", "dif"):
            for t in sp.matrix_tiles:
                if t <= half and half % t == 0 and (t <= 4096 or (t == half and 13 <= l - 1 <= 16)) and t >= 64:
                    cands[f"h_{core_dir}_t{t}"] = _desc(flow, "matrix-resident", "dense-dot-fft64",
                                                        {"real_flow": flow, "tile": t, "rows": 1,
                                                         "variant": "spread", "batch": b},
                                                        executed=f"fft_{core_dir}_matrix_batch")
        return cands, [f"m4_folded_{d}"]
    if b == 1:
        cands[f"m0_{d}"] = _desc("baseline-global-stage", "global-stage", "radix2-scalar", {})
        cands[f"m5_r4_{d}"] = _desc("baseline-global-stage", "global-stage", "radix4-scalar", {"radix": 4})
        if d == "dit":
            for t in sp.fused_tile_candidates:
                if 1 < t <= n and t <= 4096 and t >= 16:
                    cands[f"m1_t{t}"] = _desc("local-fused-tile", "fused-inplace", "radix2-scalar", {"tile": t})
        incumbents = [f"m0_{d}"]
    else:
        for v in ("spread", "folded"):
            cands[f"m4_{v}_{d}"] = _desc(f"batch-{v}", "global-stage", "radix2-scalar", {"variant": v, "batch": b})
        cands[f"m5_r4_{d}"] = _desc("batch-spread", "global-stage", "radix4-scalar",
                                    {"radix": 4, "variant": "spread", "batch": b})
        incumbents = [f"m4_spread_{d}", f"m4_folded_{d}"]
    for t in sp.matrix_tiles:
        # tile = N: one HBM round trip -- the fused single pass for 2^13..2^20
        # with a batch, the cluster kernel for 2^13..2^16 at batch 1
        if t <= n and n % t == 0 and (t <= 4096 or (t == n and (13 <= l <= 16 or (l <= 20 and b > 1)))):
            params = {"tile": t, "rows": 1}
            if b > 1:
                params.update(variant="spread", batch=b)
            cands[f"m2_{d}_t{t}"] = _desc("local-fused-tile", "matrix-resident", "dense-dot-fft64", params)
    if b == 1 and n >= 256:
        cands[f"m3_g_{d}_t64"] = _desc("local-fused-tile", "grouped-boundary", "composite-linear-map",
                                       {"tile": 64, "glog": 4, "maxp": 65536, "cells": 1})
    # exact-shape composition candidates (the 4-step run_hybrid flow, both
    # factors CTA-resident): measured beside the table candidates, promoted
    # only through the composition table (compose), never a table entry
    if d == "dit" and shape.transform_type == "c2c" and shape.transform_direction == "forward" \
            and shape.normalization == "backward" and not shape.semantic:
        t = max(16, n // 4096)
        while t <= min(4096, n // 16):
            cands[f"hyb_t{t}"] = {"block": 256, "flow_id": "hybrid-4step",
                                  "flow_realization": "decomposition-composition",
                                  "processing_unit": "b200-pass-subfft", "params": {"tile": t, "core": "b200-pass"},
                                  "executed": "run_hybrid", "composition": True}
            t *= 2
    return cands, incumbents


def _plan_of(shape: Shape, desc: dict):
    """ExecutionPlan that runs one candidate descriptor."""
    from .entry import ExecutionPlan, _dispatch
    from .selector import Selection

    params = dict(desc["params"])
    name = desc.get("executed")
    if desc.get("composition"):
        params["flow_kind"] = "composition"
    if name is None:
        sel = Selection(n=shape.n, direction=shape.direction, batch=shape.batch, precision="fp32", source="table",
                        reason="candidate", block=desc["block"], flow_id=desc["flow_id"],
                        flow_realization=desc["flow_realization"], processing_unit=desc["processing_unit"],
                        params=params)
        name = _dispatch(sel)
    if name is None:
        raise ConfigError(f"candidate {desc} has no lowering")
    return ExecutionPlan(n=shape.n, batch=shape.batch, direction=shape.direction, precision="fp32",
                         selection_source="table", reason="table-builder candidate", fallback=False,
                         executed=name, block=desc["block"], flow_id=desc["flow_id"],
                         flow_realization=desc["flow_realization"], processing_unit=desc["processing_unit"],
                         params=params, transform_type=shape.transform_type,
                         transform_direction=shape.transform_direction, norm=shape.normalization)


# ---------------------------------------------------------------- measurement (GPU)

def _reference_rows(shape: Shape, x_rows):
    import numpy as np

    nm = shape.normalization
    xd = x_rows.astype(np.complex128) if shape.transform_type != "r2c" else x_rows.astype(np.float64)
    if shape.transform_type == "r2c":
        return np.fft.rfft(xd, axis=-1, norm=nm if nm != "none" else "backward")
    if shape.transform_type == "c2r":
        return np.fft.irfft(xd, n=shape.n, axis=-1, norm=nm if nm != "none" else "forward")
    if shape.transform_direction == "forward":
        return np.fft.fft(xd, axis=-1, norm=nm if nm != "none" else "backward")
    return np.fft.ifft(xd, axis=-1, norm=nm if nm != "none" else "forward")


def _input(shape: Shape, device, seed: int):
    import numpy as np
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    b, n = shape.batch, shape.n
    if shape.transform_type == "r2c":
        x = torch.randn(b, n, device=device, generator=g)
    elif shape.transform_type == "c2r":
        # a Hermitian half spectrum: rfft of real data
        r = np.random.default_rng(seed).standard_normal((b, n))
        x = torch.from_numpy(np.fft.rfft(r, axis=-1).astype(np.complex64)).to(device)
    else:
        x = torch.complex(torch.randn(b, n, device=device, generator=g), torch.randn(b, n, device=device, generator=g))
    return x[0].contiguous() if b == 1 else x


def _spin_cycles() -> int:
    return 400_000  # ~0.2 ms at B200 clocks: longer than one call's host enqueue


def measure(shapes: list[Shape] | None = None, *, sessions: int = 3, trials: int = 20, warmup: int = 5,
            threshold: float = DEFAULT_THRESHOLD, device: int = 0, seed: int = 1234, log=None) -> dict:
    """Time every candidate of every shape on ``device``; returns the run dict."""
    import numpy as np
    import torch

    from .entry import execute_fft_plan
    from .envcheck import collect, env_hash

    shapes = shapes if shapes is not None else default_shapes()
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    env = collect(device)
    props = torch.cuda.get_device_properties(device)
    manifest = {
        "device": props.name, "profile_hash": DeviceProfile.load().hash(), "env_hash": env_hash(env), "env": env,
        "device_identity": {"device_model": props.name, "multiprocessor_count": int(props.multi_processor_count),
                            "max_shared_mem": int(getattr(props, "shared_memory_per_block_optin", 0))},
        "precision": "fp32", "dtype": "complex64", "correctness_threshold": threshold, "warmup": warmup,
        "trials": trials, "sessions": sessions, "timing_scope": TIMING_SCOPE, "protocol_id": PROTOCOL_ID,
        "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
    }
    if manifest["env_hash"] is None:
        raise RuntimeError("environment fingerprint unknown; a table measured here could never be selected")
    stream = torch.cuda.current_stream(dev)
    rng = random.Random(seed)
    out_shapes = []
    for si, shape in enumerate(shapes):
        cands, incumbents = candidates(shape)
        x = _input(shape, dev, seed + si)
        rows = sorted({0, shape.batch // 2, shape.batch - 1})
        xr = x.unsqueeze(0) if shape.batch == 1 else x
        ref = _reference_rows(shape, xr[rows].cpu().numpy())
        rec = {"key": shape.key, **shape.as_dict(), "incumbents": incumbents, "candidates": {}, "extras_failed": []}
        plans = {}
        for name, desc in cands.items():
            try:
                plan = _plan_of(shape, desc)
                y = execute_fft_plan(plan, x)
                yr = (y.unsqueeze(0) if shape.batch == 1 else y)[rows].cpu().numpy().astype(
                    np.float64 if shape.transform_type == "c2r" else np.complex128)
                err = max(float(np.linalg.norm(yr[i] - ref[i]) / max(np.linalg.norm(ref[i]), 1e-300))
                          for i in range(len(rows)))
                for _ in range(warmup):
                    execute_fft_plan(plan, x)
                plans[name] = plan
                rec["candidates"][name] = {"descriptor": desc, "executed": plan.executed, "err_max": err,
                                           "session_medians_ms": [], "n_trials": 0}
            except Exception as e:  # noqa: BLE001 - recorded, never silently skipped
                rec["extras_failed"].append({"candidate": name, "error": f"{type(e).__name__}: {e}"})
        torch.cuda.synchronize(dev)
        for s in range(sessions):
            order = list(plans)
            rng.shuffle(order)
            for name in order:
                plan = plans[name]
                times = []
                for _ in range(trials):
                    st = torch.cuda.Event(enable_timing=True)
                    en = torch.cuda.Event(enable_timing=True)
                    torch.cuda._sleep(_spin_cycles())
                    st.record(stream)
                    execute_fft_plan(plan, x)
                    en.record(stream)
                    en.synchronize()
                    times.append(st.elapsed_time(en))
                c = rec["candidates"][name]
                c["session_medians_ms"].append(statistics.median(times))
                c["n_trials"] += len(times)
        for name, c in rec["candidates"].items():
            c["sessions"] = len(c["session_medians_ms"])
            c["median_ms"] = statistics.median(c["session_medians_ms"]) if c["session_medians_ms"] else None
            c["complete"] = c["sessions"] == sessions and c["n_trials"] == sessions * trials
        # independent confirmation session: the best composition candidate and
        # the best table candidate, timed again after the search sessions
        conf = {}
        for comp in (True, False):
            pool = [(c["median_ms"], k) for k, c in rec["candidates"].items()
                    if c["median_ms"] and bool(c["descriptor"].get("composition")) == comp]
            if not pool:
                continue
            name = min(pool)[1]
            times = []
            for _ in range(trials):
                st = torch.cuda.Event(enable_timing=True)
                en = torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(_spin_cycles())
                st.record(stream)
                execute_fft_plan(plans[name], x)
                en.record(stream)
                en.synchronize()
                times.append(st.elapsed_time(en))
            times.sort()
            p50 = statistics.median(times)
            conf[name] = {"p50_ms": p50, "mad_ms": statistics.median(abs(t - p50) for t in times),
                          "p95_ms": times[min(len(times) - 1, int(0.95 * len(times)))], "trials": len(times)}
        rec["confirmation"] = conf
        out_shapes.append(rec)
        if log:
            best = min((c["median_ms"], k) for k, c in rec["candidates"].items() if c["median_ms"])
            log(f"[{si + 1}/{len(shapes)}] {shape.key}: {len(rec['candidates'])} candidates, best {best[1]} "
                f"{best[0]:.4f} ms, failed {len(rec['extras_failed'])}")
        del x
    return {"schema": "bfft-selector-run-v1", "manifest": manifest, "shapes": out_shapes}


# ---------------------------------------------------------------- gates and build (host only)

def _finite_positive(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v) and v > 0


def candidate_verdict(shape: dict, name: str, *, threshold: float, sessions: int, trials: int) -> tuple:
    """(median_ms, None) when ``name`` may be compared, else (None, reason).

    Complete-evidence rule of the reference (src/xpu/evidence.py:25-67):
    present, no recorded failure, complete flag, finite positive median,
    finite error below the threshold, every session and trial present."""
    where = f"{shape.get('key')} {name}"
    cand = (shape.get("candidates") or {}).get(name)
    if cand is None:
        return None, f"{where}: absent from the session set (incomplete evidence; cannot promote)"
    if name in {f.get("candidate") for f in shape.get("extras_failed") or ()}:
        return None, f"{where}: recorded failure in a session (extras_failed); cannot promote"
    if cand.get("complete") is not True:
        return None, f"{where}: complete evidence flag not true ({cand.get('complete')!r}); cannot promote"
    ms = cand.get("median_ms")
    if not _finite_positive(ms):
        return None, f"{where}: median not finite positive ({ms!r})"
    err = cand.get("err_max")
    if not isinstance(err, (int, float)) or not math.isfinite(err):
        return None, f"{where}: missing/non-finite error ({err!r})"
    if err >= threshold:
        return None, f"{where}: max_rel_error {err:.3e} >= {threshold:g}"
    if cand.get("sessions") != sessions:
        return None, f"{where}: session evidence {cand.get('sessions')!r}/{sessions} incomplete; cannot promote"
    if cand.get("n_trials") != sessions * trials:
        return None, f"{where}: trial evidence {cand.get('n_trials')!r}/{sessions * trials} incomplete; cannot promote"
    if any(not _finite_positive(v) for v in cand.get("session_medians_ms") or [None]):
        return None, f"{where}: a session median is not finite positive"
    return ms, None


def _sha256_of(obj) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _entry(shape: dict, desc: dict, inc_name: str, inc_ms: float, inc_block: int, ch_name: str, ch_ms: float,
           gain: float, reason: str) -> dict:
    e = {"N": shape["n"], "batch": shape["batch"], "direction": shape["direction"]}
    if shape.get("semantic"):
        e.update(transform_type=shape["transform_type"], transform_direction=shape["transform_direction"],
                 normalization=shape["normalization"])
    e.update(incumbent_ms=inc_ms, incumbent_block=inc_block, challenger_ms=ch_ms,
             evidence={"incumbent": f"{inc_name}@block{inc_block}",
                       "challenger": f"{ch_name}@block{desc['block']}", "gain_pct": round(gain, 3)},
             reason=reason, block=desc["block"], flow_id=desc["flow_id"],
             flow_realization=desc["flow_realization"], processing_unit=desc["processing_unit"],
             params=dict(desc["params"]))
    if desc.get("executed"):
        e["executed"] = desc["executed"]
    return e


def build_table(runs: list[dict], *, guard_pct: float = GUARD_PCT, sources: list[str] | None = None) -> dict:
    """Selector table from measured runs (raises ConfigError when the result
    would not load)."""
    if not runs:
        raise ConfigError("no runs to build from")
    rejections: list[str] = []
    base = runs[0].get("manifest") or {}
    for k in MANIFEST_KEYS:
        if base.get(k) in (None, ""):
            raise ConfigError(f"run 0 manifest missing {k!r}")
    accepted = [runs[0]]
    for i, r in enumerate(runs[1:], 1):
        m = r.get("manifest") or {}
        diff = [k for k in MANIFEST_KEYS if m.get(k) != base.get(k)]
        if diff:
            rejections.append(f"run {i}: manifest differs from run 0 in {', '.join(diff)}; run refused")
        else:
            accepted.append(r)
    shapes: dict[str, dict] = {}
    for r in accepted:
        for s in r.get("shapes") or ():
            shapes[s["key"]] = s  # a later run re-measures the shape
    thr, ns, nt = float(base["correctness_threshold"]), int(base["sessions"]), int(base["trials"])
    entries = []
    for key in sorted(shapes, key=lambda k: (shapes[k]["semantic"], shapes[k]["n"], shapes[k]["batch"],
                                             shapes[k]["direction"], k)):
        s = shapes[key]
        verdicts = {}
        for name in s.get("candidates") or {}:
            if s["candidates"][name]["descriptor"].get("composition"):
                continue  # promoted only through the composition table
            ms, why = candidate_verdict(s, name, threshold=thr, sessions=ns, trials=nt)
            if why:
                rejections.append(why)
            else:
                verdicts[name] = ms
        for f in s.get("extras_failed") or ():
            rejections.append(f"{key} {f.get('candidate')}: failed to run ({f.get('error')})")
        incs = [(verdicts[i], i) for i in s.get("incumbents") or () if i in verdicts]
        if not incs:
            rejections.append(f"{key}: no admissible incumbent ({s.get('incumbents')}); no entry")
            continue
        inc_ms, inc = min(incs)
        inc_desc = s["candidates"][inc]["descriptor"]
        chal = [(ms, n) for n, ms in verdicts.items() if n not in (s.get("incumbents") or ())]
        if chal:
            ch_ms, ch = min(chal)
            gain = (inc_ms - ch_ms) / inc_ms * 100.0
        else:
            ch_ms, ch, gain = None, None, float("-inf")
        if ch is not None and gain >= guard_pct:
            desc = s["candidates"][ch]["descriptor"]
            reason = f"challenger {ch}@block{desc['block']} beats incumbent {inc}@block{inc_desc['block']} " \
                     f"by {gain:.1f}% (>= {guard_pct}%)"
            entries.append(_entry(s, desc, inc, inc_ms, inc_desc["block"], ch, ch_ms, gain, reason))
        elif s["batch"] > 1 and inc.startswith("m4_") and not s.get("semantic"):
            other = [i for i in s.get("incumbents") or () if i != inc and i in verdicts]
            vs = f" over {other[0]} ({verdicts[other[0]]:.4f} ms)" if other else ""
            note = f"; best challenger {ch} gains {gain:.1f}% < {guard_pct}%" if ch else ""
            reason = f"faster M4 variant {inc}{vs}{note}"
            entries.append(_entry(s, inc_desc, inc, inc_ms, inc_desc["block"], inc, inc_ms, 0.0, reason))
        else:
            rejections.append(f"{key}: best challenger {ch} gains {gain:.1f}% < {guard_pct}% over {inc}; "
                              "no entry (M0 stays)" if ch else f"{key}: no admissible challenger; no entry")
    ident = base.get("device_identity") or {}
    table = {
        "schema_version": 2, "device": "nvidia-b200", "profile_hash": base["profile_hash"],
        "env_hash": base["env_hash"], "env": {**(base.get("env") or {}), **ident},
        "precision": base["precision"], "guard_pct": guard_pct, "selection_semantics": SELECTION_SEMANTICS,
        "protocol_id": base["protocol_id"], "correctness_threshold": thr,
        "sources": [{"path": p, "sha256": _sha256_of(r)} for p, r in zip(sources or [f"run{i}" for i in range(len(runs))],
                                                                         runs)],
        "rejections": rejections, "entries": entries,
    }
    bad = validate_table(table)
    if bad:
        raise ConfigError(f"built table violates the contract ({len(bad)}): " + "; ".join(bad[:6]))
    return table


# ---------------------------------------------------------------- composition promotion

def _git_commit() -> str:
    import subprocess

    try:
        return subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True, timeout=10,
                              cwd=os.path.dirname(os.path.abspath(__file__))).stdout.strip() or "unknown"
    except Exception:  # noqa: BLE001
        return "unknown"


def build_composition_table(runs: list[dict], selector_table: dict, *, guard_pct: float = GUARD_PCT,
                            sources: list[str] | None = None) -> tuple[dict | None, list[str]]:
    """Exact-shape composition promotions (the reference's composition
    registry, src/xpu/composition.py:59-240, config/composition_table.json).

    For every measured c2c shape the incumbent is the lowering the selector
    table chose for it (M0 / the faster M4 variant when the table has no
    entry), timed in the same run; the best admissible 4-step candidate is
    promoted when it beats the incumbent by at least the guard in the search
    sessions and was re-timed in the independent confirmation session.
    Returns (table or None when nothing is promoted, verdict lines)."""
    from . import _build
    from .composition import KIND, rows_sha256, table_violations
    from .selector import find_entry

    base = runs[0]["manifest"]
    thr, ns, nt = float(base["correctness_threshold"]), int(base["sessions"]), int(base["trials"])
    names = sources or [f"run{i}" for i in range(len(runs))]
    notes, entries = [], []
    for ri, run in enumerate(runs):
        if any(run["manifest"].get(k) != base.get(k) for k in MANIFEST_KEYS):
            notes.append(f"run {ri}: manifest differs from run 0; refused")
            continue
        for s in run["shapes"]:
            comps = [k for k, c in s["candidates"].items() if c["descriptor"].get("composition")]
            if not comps:
                continue
            key = s["key"]
            e = find_entry(selector_table, s["n"], s["batch"], s["direction"])
            if e is not None and e.get("evidence"):
                inc = e["evidence"]["challenger"].split("@")[0]
            else:
                incs = [(s["candidates"][i]["median_ms"], i) for i in s.get("incumbents") or ()
                        if s["candidates"].get(i, {}).get("median_ms")]
                inc = min(incs)[1] if incs else None
            inc_ms, why = (None, "no incumbent") if inc is None else \
                candidate_verdict(s, inc, threshold=thr, sessions=ns, trials=nt)
            if why:
                notes.append(f"{key}: incumbent {inc}: {why}; no promotion")
                continue
            best = None
            for k in comps:
                ms, why = candidate_verdict(s, k, threshold=thr, sessions=ns, trials=nt)
                if why:
                    notes.append(why)
                elif best is None or ms < best[0]:
                    best = (ms, k)
            if best is None:
                continue
            gain = (inc_ms - best[0]) / inc_ms * 100.0
            conf = (s.get("confirmation") or {}).get(best[1])
            if gain < guard_pct:
                notes.append(f"{key}: best 4-step {best[1]} {best[0]:.4f} ms vs incumbent {inc} {inc_ms:.4f} ms "
                             f"({gain:+.1f}% < {guard_pct}%); not promoted")
                continue
            if not conf:
                notes.append(f"{key}: {best[1]} passes the guard but has no confirmation session; not promoted")
                continue
            c = s["candidates"][best[1]]
            entries.append({
                "N": s["n"], "batch": s["batch"], "direction": "dit", "precision": "fp32",
                "tile": int(c["descriptor"]["params"]["tile"]), "core": "b200-pass", "flow_id": "hybrid-4step",
                "flow_realization": "decomposition-composition", "processing_unit": "b200-pass-subfft",
                "candidate_ms": best[0], "incumbent_ms": inc_ms, "incumbent_flow": inc,
                "guard_pct": guard_pct_value(best[0], inc_ms), "guard_pass": True,
                "reason": f"exact-shape 4-step {best[1]} {best[0]:.4f} ms vs table winner {inc} {inc_ms:.4f} ms "
                          f"(+{gain:.1f}%)",
                "evidence": {"artifact": names[ri], "artifact_sha256": _sha256_of(run), "commit": _git_commit(),
                             "sessions": ns, "trials": nt, "confirmation_session": True, "err_max": c["err_max"],
                             "p50_ms": conf["p50_ms"], "mad_ms": conf["mad_ms"], "p95_ms": conf["p95_ms"]}})
            notes.append(f"{key}: promoted {best[1]} (+{gain:.1f}% over {inc})")
    if not entries:
        return None, notes
    table = {"schema_version": 1, "kind": KIND, "profile_hash": base["profile_hash"], "env_hash": base["env_hash"],
             "precision": "fp32", "guard_pct": guard_pct, "contract_id": "b200_pass_core", "entries": entries,
             "source_hash": _build.source_hash(), "result_sha256": rows_sha256({"rows": entries}),
             "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}
    bad = table_violations(table)
    if bad:
        raise ConfigError(f"built composition table violates its contract ({len(bad)}): " + "; ".join(bad[:6]))
    return table, notes


def guard_pct_value(candidate_ms: float, incumbent_ms: float) -> float:
    from .composition import guard_pct_of

    return guard_pct_of(candidate_ms, incumbent_ms)


# ---------------------------------------------------------------- run files

def save_run(run: dict, path: str) -> None:
    """Write a run file (gzip-compressed when ``path`` ends in .gz)."""
    import gzip

    blob = json.dumps(run, separators=(",", ":")).encode()
    if path.endswith(".gz"):
        with gzip.open(path, "wb", compresslevel=9) as f:
            f.write(blob)
    else:
        with open(path, "wb") as f:
            f.write(blob)


def load_run(path: str) -> dict:
    import gzip

    opener = gzip.open if path.endswith(".gz") else open
    with opener(path, "rb") as f:
        return json.loads(f.read().decode())


# ---------------------------------------------------------------- CLI

def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m bfft.table_builder")
    sub = ap.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("measure", help="time every candidate of the size matrix on a B200")
    m.add_argument("--out", required=True)
    m.add_argument("--quick", action="store_true")
    m.add_argument("--sessions", type=int, default=3)
    m.add_argument("--trials", type=int, default=20)
    m.add_argument("--warmup", type=int, default=5)
    m.add_argument("--device", type=int, default=0)
    m.add_argument("--only", nargs="+", default=None, metavar="KEY",
                   help="measure only these shape keys (e.g. N1048576B16:dit:c2c-forward-backward); "
                        "build merges runs, a later run re-measuring its shapes")
    b = sub.add_parser("build", help="build the selector table from run files")
    b.add_argument("runs", nargs="+")
    b.add_argument("--out", default=TABLE_PATH)
    b.add_argument("--guard-pct", type=float, default=GUARD_PCT)
    c = sub.add_parser("compose", help="promote exact-shape 4-step compositions from run files")
    c.add_argument("runs", nargs="+")
    c.add_argument("--selector", default=TABLE_PATH)
    c.add_argument("--out", default=None)
    c.add_argument("--guard-pct", type=float, default=GUARD_PCT)
    a = ap.parse_args(argv)
    if a.cmd == "measure":
        shapes = default_shapes(a.quick)
        if a.only:
            known = {s.key for s in shapes}
            unknown = [k for k in a.only if k not in known]
            if unknown:
                raise ConfigError(f"--only: not shapes of the size matrix: {', '.join(unknown)}")
            shapes = [s for s in shapes if s.key in set(a.only)]
        run = measure(shapes, sessions=a.sessions, trials=a.trials, warmup=a.warmup,
                      device=a.device, log=lambda s: print(s, file=sys.stderr, flush=True))
        save_run(run, a.out)
        return 0
    runs = [load_run(p) for p in a.runs]
    if a.cmd == "compose":
        from .composition import TABLE_PATH as COMP_PATH
        from .selector import load_table

        table, notes = build_composition_table(runs, load_table(a.selector), guard_pct=a.guard_pct,
                                               sources=[os.path.basename(p) for p in a.runs])
        for line in notes:
            print(line)
        out = a.out or COMP_PATH
        if table is None:
            print(f"no composition promoted; {out} not written")
            return 0
        with open(out, "w") as f:
            json.dump(table, f, indent=1)
            f.write("\n")
        print(f"{len(table['entries'])} composition entries -> {out}")
        return 0
    table = build_table(runs, guard_pct=a.guard_pct, sources=[os.path.basename(p) for p in a.runs])
    with open(a.out, "w") as f:
        json.dump(table, f, indent=1)
        f.write("\n")
    print(f"{len(table['entries'])} entries, {len(table['rejections'])} rejections -> {a.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
