"""Selector table builder: candidate enumeration, evidence gates, the promotion
guard, manifest binding, and that a built table loads and selects (no GPU;
synthetic run files stand in for B200 measurements)."""
import copy

import pytest

from bfft import table_builder as TB
from bfft.config import ConfigError, DeviceProfile
from bfft.selector import select, validate_table

ENV = "0123456789abcdef"


def _manifest(**kw):
    m = {"device": "NVIDIA B200", "profile_hash": DeviceProfile.load().hash(), "env_hash": ENV,
         "env": {"device_name": "NVIDIA B200"},
         "device_identity": {"device_model": "NVIDIA B200", "multiprocessor_count": 148, "max_shared_mem": 232448},
         "precision": "fp32", "dtype": "complex64", "correctness_threshold": 1e-6, "warmup": 5, "trials": 20,
         "sessions": 3, "timing_scope": TB.TIMING_SCOPE, "protocol_id": TB.PROTOCOL_ID}
    m.update(kw)
    return m


def _shape_rec(shape: TB.Shape, times: dict, errs: dict | None = None, sessions=3, trials=20):
    cands, incs = TB.candidates(shape)
    rec = {"key": shape.key, **shape.as_dict(), "incumbents": incs, "candidates": {}, "extras_failed": []}
    for name, ms in times.items():
        rec["candidates"][name] = {"descriptor": cands[name], "executed": None,
                                   "err_max": (errs or {}).get(name, 2e-7),
                                   "session_medians_ms": [ms] * sessions, "n_trials": sessions * trials,
                                   "sessions": sessions, "median_ms": ms, "complete": True}
    return rec


def _run(recs, **mkw):
    return {"schema": "bfft-selector-run-v1", "manifest": _manifest(**mkw), "shapes": recs}


def test_candidate_enumeration_matches_the_design_space():
    c, inc = TB.candidates(TB.Shape(2048, 1, "dit"))
    assert inc == ["m0_dit"] and "m0_dit" in c and "m5_r4_dit" in c
    assert "m1_t64" in c and "m2_dit_t2048" in c and "m2_dit_t4096" not in c
    c, inc = TB.candidates(TB.Shape(65536, 1, "dif"))
    assert "m2_dif_t65536" in c and not any(k.startswith("m1_") for k in c)  # cluster tile, no DIF M1
    c, inc = TB.candidates(TB.Shape(1 << 20, 16, "dit"))  # the fused single pass (tile = N) with a batch
    assert inc == ["m4_spread_dit", "m4_folded_dit"] and "m2_dit_t1024" in c and "m2_dit_t1048576" in c
    c, _ = TB.candidates(TB.Shape(1 << 20, 1, "dit"))  # no single-pass kernel for one 2^20 transform
    assert "m2_dit_t1024" in c and "m2_dit_t1048576" not in c
    c, inc = TB.candidates(TB.Shape(4096, 256, "dit", "r2c", "forward", "backward", True))
    assert inc == ["m4_folded_dit"] and c["h_dif_t2048"]["executed"] == "fft_dif_matrix_batch"
    c, _ = TB.candidates(TB.Shape(2048, 16, "dit"))
    assert {k for k in c if k.startswith("hyb_")} == {"hyb_t16", "hyb_t32", "hyb_t64", "hyb_t128"}
    for shape in TB.default_shapes():
        for desc in TB.candidates(shape)[0].values():
            if desc.get("composition"):
                continue  # composition candidates are promoted through their own table
            e = {"N": shape.n, "batch": shape.batch, "direction": shape.direction, **desc}
            from bfft.selector import entry_contract_violations

            assert entry_contract_violations(e) == [], (shape.key, desc)


def test_guard_and_gates():
    s1 = TB.Shape(1024, 1, "dit")
    s2 = TB.Shape(2048, 1, "dit")
    s3 = TB.Shape(4096, 1, "dif")
    recs = [
        _shape_rec(s1, {"m0_dit": 1.0, "m2_dit_t1024": 0.979}),          # 2.1% -> entry
        _shape_rec(s2, {"m0_dit": 1.0, "m2_dit_t2048": 0.981}),          # 1.9% -> no entry
        _shape_rec(s3, {"m0_dif": 1.0, "m2_dif_t4096": 0.5, "m5_r4_dif": 0.9},
                   errs={"m2_dif_t4096": 3e-6}),                            # error gate -> r4 wins
    ]
    t = TB.build_table([_run(recs)])
    assert validate_table(t) == []
    keys = {(e["N"], e["direction"]): e for e in t["entries"]}
    assert keys[(1024, "dit")]["params"]["tile"] == 1024
    assert (2048, "dit") not in keys
    assert keys[(4096, "dif")]["processing_unit"] == "radix4-scalar"
    assert any("max_rel_error" in r for r in t["rejections"])
    assert any("1.9%" in r for r in t["rejections"])


def test_incomplete_evidence_is_refused():
    s = TB.Shape(1024, 1, "dit")
    rec = _shape_rec(s, {"m0_dit": 1.0, "m2_dit_t1024": 0.5, "m5_r4_dit": 0.8})
    rec["candidates"]["m2_dit_t1024"]["n_trials"] = 59
    rec["extras_failed"].append({"candidate": "m5_r4_dit", "error": "boom"})
    t = TB.build_table([_run([rec])])
    assert t["entries"] == []
    assert any("trial evidence" in r for r in t["rejections"])
    assert any("extras_failed" in r for r in t["rejections"])
    rec2 = _shape_rec(s, {"m0_dit": float("nan"), "m2_dit_t1024": 0.5})
    t2 = TB.build_table([_run([rec2])])
    assert t2["entries"] == [] and any("no admissible incumbent" in r for r in t2["rejections"])


def test_batched_keeps_faster_m4_variant():
    s = TB.Shape(4096, 4096, "dit")
    t = TB.build_table([_run([_shape_rec(s, {"m4_spread_dit": 2.0, "m4_folded_dit": 1.5, "m2_dit_t4096": 1.49})])])
    (e,) = t["entries"]
    assert e["flow_id"] == "batch-folded" and e["params"]["variant"] == "folded"
    t = TB.build_table([_run([_shape_rec(s, {"m4_spread_dit": 2.0, "m4_folded_dit": 1.5, "m2_dit_t4096": 0.4})])])
    (e,) = t["entries"]
    assert e["flow_realization"] == "matrix-resident" and e["evidence"]["incumbent"].startswith("m4_folded")


def test_manifest_mismatch_refuses_run():
    s = TB.Shape(1024, 1, "dit")
    good = _run([_shape_rec(s, {"m0_dit": 1.0, "m2_dit_t1024": 0.5})])
    other = _run([_shape_rec(TB.Shape(2048, 1, "dit"), {"m0_dit": 1.0, "m2_dit_t2048": 0.5})], env_hash="ffff")
    t = TB.build_table([good, other])
    assert len(t["entries"]) == 1 and any("manifest differs" in r for r in t["rejections"])
    bad = copy.deepcopy(good)
    del bad["manifest"]["protocol_id"]
    with pytest.raises(ConfigError):
        TB.build_table([bad])


def test_built_table_selects_through_the_selector():
    recs = [_shape_rec(TB.Shape(1024, 1, "dit"), {"m0_dit": 1.0, "m2_dit_t1024": 0.3}),
            _shape_rec(TB.Shape(4096, 256, "dit", "r2c", "forward", "backward", True),
                       {"m4_folded_dit": 3.0, "h_dif_t2048": 0.7, "h_dit_t2048": 0.8})]
    t = TB.build_table([_run(recs)])
    ph = DeviceProfile.load().hash()
    sel = select("dit", 1024, profile_hash=ph, table=t, env_hash=ENV)
    assert sel.selected and sel.params["tile"] == 1024
    assert not select("dit", 1024, profile_hash=ph, table=t, env_hash="0" * 16).selected
    sel = select("dit", 4096, batch=256, profile_hash=ph, table=t, env_hash=ENV, transform_type="r2c")
    assert sel.selected and sel.executed == "fft_dif_matrix_batch" and sel.params["real_flow"] == "dedicated-r2c-pack-v1"
    from bfft.entry import plan_fft

    p = plan_fft("dit", 4096, batch=256, profile_hash=ph, table=t, env_hash=ENV, transform_type="r2c")
    assert not p.fallback and p.executed == "fft_dif_matrix_batch" and p.params["real_compat"]


def _with_conf(rec, name, ms):
    rec["confirmation"] = {name: {"p50_ms": ms, "mad_ms": 0.001, "p95_ms": ms * 1.05, "trials": 20}}
    return rec


def test_composition_promotion():
    from bfft.composition import composition_select, table_violations

    s1 = TB.Shape(2048, 16, "dit")
    s2 = TB.Shape(4096, 16, "dit")
    r1 = _with_conf(_shape_rec(s1, {"m4_spread_dit": 1.0, "m4_folded_dit": 0.9, "m2_dit_t2048": 0.2,
                                    "hyb_t64": 0.15, "hyb_t32": 0.3}), "hyb_t64", 0.151)
    r2 = _shape_rec(s2, {"m4_spread_dit": 1.0, "m4_folded_dit": 0.9, "m2_dit_t4096": 0.2, "hyb_t64": 0.199})
    run = _run([r1, r2])
    sel = TB.build_table([run])
    assert all(e["flow_id"] != "hybrid-4step" for e in sel["entries"])  # never a selector entry
    table, notes = TB.build_composition_table([run], sel, sources=["run.json.gz"])
    assert table is not None and len(table["entries"]) == 1
    e = table["entries"][0]
    assert (e["N"], e["batch"], e["tile"], e["incumbent_flow"]) == (2048, 16, 64, "m2_dit_t2048")
    assert abs(e["guard_pct"] - 25.0) < 1e-9 and e["evidence"]["confirmation_session"]
    assert table_violations(table) == []
    assert any("0.5%" in n or "not promoted" in n for n in notes)  # 4096: +0.5% < guard
    ph = DeviceProfile.load().hash()
    assert composition_select("dit", 2048, batch=16, profile_hash=ph, env_hash=ENV, table=table)["tile"] == 64
    assert composition_select("dit", 2048, batch=16, profile_hash=ph, env_hash="f" * 16, table=table) is None
    # no confirmation session -> no promotion
    r3 = _shape_rec(s1, {"m4_spread_dit": 1.0, "m4_folded_dit": 0.9, "m2_dit_t2048": 0.2, "hyb_t64": 0.1})
    t3, notes3 = TB.build_composition_table([_run([r3])], sel)
    assert t3 is None and any("confirmation" in n for n in notes3)
