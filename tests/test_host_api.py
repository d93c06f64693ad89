"""Host-side API semantics (no GPU): plan resolution, selector gates,
composition contract, input contracts, config loaders, tail partition.

The plan-semantics cases replay queries that were run against the reference's
own plan_fft on a synthetic table (tests/golden/make_golden.py) and require
identical plan fields: executed runner, fallback flag, selection source,
reason, block, attribution and params.
"""
import copy
import json
import math

import numpy as np
import pytest

import bfft
from bfft import entry, selector
from bfft.candidates import Candidate, check_lowering
from bfft.composition import composition_select, guard_pct_of, load_composition_table, rows_sha256
from bfft.config import ConfigError, DesignSpace, DeviceProfile, SizeMatrix
from bfft.entry import ExecutionPlan, _check_plan_input, norm_scale, plan_fft
from bfft.matrices import local_matrix, tail_groups

PLAN_FIELDS = ("n", "batch", "direction", "precision", "selection_source", "reason", "fallback",
               "executed", "block", "flow_id", "flow_realization", "processing_unit", "params",
               "transform_type", "transform_direction", "norm")


def test_plan_semantics_match_reference_on_synthetic_table(golden_meta):
    table = golden_meta["synthetic_table"]
    checked = 0
    for label, rec in golden_meta["plans"].items():
        q = dict(rec["query"])
        if rec.get("raises") is not None:
            with pytest.raises(ValueError):
                plan_fft(table=copy.deepcopy(table), profile_hash="p-synth-0001",
                         env_hash="e-synth-0001", **q) if label.startswith("bad-") else \
                    plan_fft(table=copy.deepcopy(table), **q)
            checked += 1
            continue
        if rec.get("raises") is None and "plan" not in rec:
            continue
        p = plan_fft(table=copy.deepcopy(table), **q)
        for f in PLAN_FIELDS:
            assert getattr(p, f) == rec["plan"][f], (label, f, getattr(p, f), rec["plan"][f])
        checked += 1
    assert checked >= 25


def test_plan_is_host_only_and_frozen():
    p = plan_fft("dit", 256, 4, profile_hash=None)
    assert p.fallback and p.selection_source == "abstain" and p.executed == "fft_dit_batch"
    assert p.params == {"variant": "folded", "batch": 4}
    with pytest.raises(Exception):
        p.n = 3  # frozen dataclass
    r = p.as_report()
    assert isinstance(r, bfft.ExecutionReport) and r.executed == p.executed


@pytest.mark.parametrize("bad", [dict(direction="fft"), dict(precision="fp16"), dict(transform_type="dct"),
                                 dict(transform_direction="up"), dict(norm="unit"),
                                 dict(transform_type="r2c", transform_direction="inverse"),
                                 dict(transform_type="c2r", transform_direction="forward")])
def test_bad_semantics_raise_before_table_query(bad, monkeypatch):
    def boom(*a, **k):
        raise AssertionError("table queried")

    monkeypatch.setattr(entry, "load_table", boom)
    monkeypatch.setattr(entry, "select", boom)
    kw = dict(direction="dit", n=256)
    kw.update(bad)
    with pytest.raises(ValueError):
        plan_fft(**kw)


def test_norm_scale_is_torch_fft_semantics():
    import torch

    x = torch.randn(64, dtype=torch.complex64)
    for norm in ("forward", "backward", "ortho"):
        f = torch.fft.fft(x, norm=norm)
        assert torch.allclose(f, torch.fft.fft(x) * norm_scale(64, "forward", norm), atol=1e-4)
        i = torch.fft.ifft(x, norm=norm)
        assert torch.allclose(i, torch.fft.ifft(x, norm="forward") * norm_scale(64, "inverse", norm), atol=1e-5)
    assert norm_scale(64, "forward", "none") == 1.0 == norm_scale(64, "inverse", "none")
    assert math.isclose(norm_scale(16, "inverse", "ortho"), 0.25)
    with pytest.raises(ValueError):
        norm_scale(8, "sideways", "none")


def _plan(**kw):
    base = dict(n=1024, batch=1, direction="dit", precision="fp32", selection_source="table",
                reason="", fallback=False, executed="fft_dit")
    base.update(kw)
    return ExecutionPlan(**base)


def test_check_plan_input_contracts():
    _check_plan_input(_plan(), (1024,), "complex64")
    with pytest.raises(TypeError):
        _check_plan_input(_plan(), (1024,), "complex128")
    with pytest.raises(ValueError):
        _check_plan_input(_plan(), (1, 1024), "complex64")
    _check_plan_input(_plan(batch=4), (4, 1024), "complex64")
    with pytest.raises(ValueError):
        _check_plan_input(_plan(batch=4), (8, 1024), "complex64")
    _check_plan_input(_plan(transform_type="r2c"), (1024,), "float32")
    with pytest.raises(TypeError):
        _check_plan_input(_plan(transform_type="r2c"), (1024,), "complex64")
    _check_plan_input(_plan(transform_type="c2r", transform_direction="inverse"), (513,), "complex64")
    with pytest.raises(ValueError):
        _check_plan_input(_plan(transform_type="c2r", transform_direction="inverse"), (1024,), "complex64")


def test_execute_rejects_non_tensor_before_launch():
    with pytest.raises(TypeError):
        bfft.execute_fft_plan(_plan(), [1, 2, 3])


def test_run_fft_rejects_bad_inputs_before_planning(monkeypatch):
    import torch

    monkeypatch.setattr(entry, "plan_fft", lambda *a, **k: (_ for _ in ()).throw(AssertionError("planned")))
    with pytest.raises(TypeError):
        bfft.run_fft(torch.zeros(8, dtype=torch.float64), "dit")
    with pytest.raises(TypeError):
        bfft.run_fft(np.zeros(8), "dit")
    with pytest.raises(ValueError):
        bfft.run_fft(torch.zeros(2, 2, 2, dtype=torch.complex64), "dit")
    with pytest.raises(ValueError):
        bfft.run_fft(torch.zeros(4, 8, dtype=torch.complex64), "dit", batch=2)
    with pytest.raises(ValueError):
        bfft.run_fft(torch.zeros(8, dtype=torch.complex64), "fft")


# ------------------------------------------------------------------ selector

def _table(tmp_path, **over):
    prof = DeviceProfile.load().hash()
    t = {"schema_version": 2, "device": "nvidia-b200", "profile_hash": prof, "env_hash": "e-test",
         "env": {"device_model": 100, "multiprocessor_count": 148, "max_shared_mem": 232448},
         "precision": "fp32", "guard_pct": 2.0,
         "entries": [{"N": 4096, "batch": 64, "direction": "dit", "block": 256, "incumbent_block": 512,
                      "flow_id": "local-fused-tile", "flow_realization": "matrix-resident",
                      "processing_unit": "dense-dot-fft64",
                      "params": {"tile": 4096, "rows": 1, "variant": "spread", "batch": 64},
                      "transform_type": "c2c", "transform_direction": "forward",
                      "normalization": "backward", "executed": "fft_dit_matrix_batch",
                      "reason": "test winner"}]}
    t.update(over)
    p = tmp_path / "selector_table.json"
    p.write_text(json.dumps(t))
    return str(p), prof


def test_selector_gates(tmp_path):
    path, prof = _table(tmp_path)
    t = selector.load_table(path)
    s = selector.select("dit", 4096, 64, profile_hash=prof, table=t, env_hash="e-test")
    assert s.selected and s.executed == "fft_dit_matrix_batch" and s.entry_tier == "semantic"
    assert not selector.select("dit", 4096, 64, profile_hash=None, table=t, env_hash="e-test").selected
    assert not selector.select("dit", 4096, 64, profile_hash="x", table=t, env_hash="e-test").selected
    assert not selector.select("dit", 4096, 64, profile_hash=prof, table=t, env_hash=None).selected
    assert not selector.select("dit", 4096, 64, profile_hash=prof, table=t, env_hash="other").selected
    assert not selector.select("dit", 4096, 32, profile_hash=prof, table=t, env_hash="e-test").selected
    assert not selector.select("dit", 4096, 64, precision="fp16", profile_hash=prof, table=t,
                               env_hash="e-test").selected
    unbound = dict(t, env_hash="")
    s2 = selector.select("dit", 4096, 64, profile_hash=prof, table=unbound, env_hash="e-test")
    assert not s2.selected and "pre-freshness" in s2.reason


def test_plan_through_b200_table(tmp_path):
    path, prof = _table(tmp_path)
    t = selector.load_table(path)
    p = plan_fft("dit", 4096, 64, profile_hash=prof, table=t, env_hash="e-test")
    assert (p.executed, p.fallback, p.selection_source) == ("fft_dit_matrix_batch", False, "table")
    q = plan_fft("dit", 4096, 64, profile_hash=prof, table=t, env_hash="e-test", norm="ortho")
    assert q.fallback and q.executed == "fft_dit_batch" and q.block == 1024


@pytest.mark.parametrize("mutate, needle", [
    (lambda e: e.update(block=100), "block"),
    (lambda e: e["params"].update(tile=1 << 21), "tile"),
    (lambda e: e["params"].update(variant="diagonal"), "variant"),
    (lambda e: e.update(executed="fft_dit"), "executed"),
    (lambda e: e.update(processing_unit="tensor-core"), "processing"),
    (lambda e: e.update(layout="planar-soa"), "layout"),
    (lambda e: e.update(transform_type="dct"), "transform_type"),
])
def test_table_contract_violations_refuse_load(tmp_path, mutate, needle):
    path, _ = _table(tmp_path)
    t = json.loads(open(path).read())
    mutate(t["entries"][0])
    with open(path, "w") as f:
        json.dump(t, f)
    with pytest.raises(ConfigError, match=needle):
        selector.load_table(path)


def test_missing_or_broken_table(tmp_path):
    with pytest.raises(ConfigError):
        selector.load_table(str(tmp_path / "nope.json"))
    p = tmp_path / "bad.json"
    p.write_text("{")
    with pytest.raises(ConfigError):
        selector.load_table(str(p))
    p.write_text(json.dumps({"entries": []}))
    with pytest.raises(ConfigError, match="profile_hash"):
        selector.load_table(str(p))


def test_previous_fallback_binding(tmp_path):
    path, prof = _table(tmp_path)
    t = json.loads(open(path).read())
    fb = copy.deepcopy(t["entries"][0])
    fb.pop("executed")
    fb["params"]["tile"] = 1024
    t["previous_fallbacks"] = [fb]
    v = selector.validate_table(t)
    assert any("previous_fallback_provenance" in m for m in v)
    fb["previous_fallback_provenance"] = {
        "carry_contract": selector.FALLBACK_CARRY_CONTRACT, "source_env_hash": "e-test",
        "source_profile_hash": prof, "source_precision": "fp32",
        "source_device": {"device_model": 100, "multiprocessor_count": 148, "max_shared_mem": 232448},
        "source_table_sha256": "x", "source_result_sha256": "y", "paired_confirm": "z"}
    assert selector.validate_table(t) == []
    s = selector.select("dit", 4096, 64, profile_hash=prof, table=t, env_hash="e-test")
    assert s.entry_tier == "previous-fallback" and s.params["tile"] == 1024
    p = plan_fft("dit", 4096, 64, profile_hash=prof, table=t, env_hash="e-test")
    assert p.params.get("previous_fallback") is True
    fb["previous_fallback_provenance"]["source_env_hash"] = "stale"
    assert any("stale evidence" in m for m in selector.validate_table(t))


def test_shipped_table_loads_and_fails_closed_without_env():
    t = selector.load_table()
    s = selector.select("dit", 4096, 64, profile_hash=DeviceProfile.load().hash(), table=t, env_hash=None)
    assert not s.selected


# ------------------------------------------------------------------ composition

def _comp_table(prof):
    e = {"N": 2048, "batch": 16, "direction": "dit", "precision": "fp32", "tile": 64, "core": "b200-pass",
         "flow_id": "hybrid-4step", "flow_realization": "composition", "processing_unit": "b200-pass",
         "candidate_ms": 0.01, "incumbent_ms": 0.02, "guard_pct": guard_pct_of(0.01, 0.02),
         "guard_pass": True, "reason": "test", "evidence": {
             "artifact": "a", "artifact_sha256": "b", "commit": "c", "sessions": 3, "trials": 10,
             "confirmation_session": "s", "err_max": 1e-7, "p50_ms": 0.01, "mad_ms": 0.0, "p95_ms": 0.01}}
    return {"schema_version": 1, "kind": "composition-promotion", "profile_hash": prof, "env_hash": "e",
            "precision": "fp32", "guard_pct": 2.0, "contract_id": "b200_pass_core", "entries": [e],
            "source_hash": "s", "result_sha256": rows_sha256({"rows": [e]})}


def test_composition_contract_and_selection(tmp_path):
    prof = DeviceProfile.load().hash()
    t = _comp_table(prof)
    p = tmp_path / "composition_table.json"
    p.write_text(json.dumps(t))
    loaded = load_composition_table(str(p))
    assert composition_select("dit", 2048, 16, profile_hash=prof, env_hash="e", table=loaded)
    assert composition_select("dif", 2048, 16, profile_hash=prof, env_hash="e", table=loaded) is None
    assert composition_select("dit", 2048, 16, profile_hash=prof, env_hash="x", table=loaded) is None
    assert composition_select("dit", 2048, 16, profile_hash=prof, env_hash="e", table=loaded,
                              transform_direction="inverse") is None
    tampered = copy.deepcopy(t)
    tampered["entries"][0]["tile"] = 128
    p.write_text(json.dumps(tampered))
    with pytest.raises(ConfigError, match="result_sha256"):
        load_composition_table(str(p))
    plan = entry._composition_plan(loaded["entries"][0], 2048, 16, "dit", "fp32", "forward", "backward")
    assert plan.executed == "run_hybrid" and plan.selection_source == "composition"
    assert plan.params["tile"] == 64 and plan.params["flow_kind"] == "composition"


# ------------------------------------------------------------------ config / contract / partition

def test_config_loaders():
    prof = DeviceProfile.load()
    assert prof.sms == 148 and prof.clusters == 148 and len(prof.hash()) == 16
    sp = DesignSpace.load()
    assert 4096 in sp.matrix_tiles and "spread" in sp.batch_variants
    assert SizeMatrix.load().correctness_sizes[0] == 2


def test_lowering_contract_cases():
    ok = Candidate(flow_id="baseline-global-stage", processing_unit="radix2-scalar", radix=2)
    assert check_lowering(ok).legal
    bad = [Candidate(flow_id="baseline-global-stage", processing_unit="radix4-scalar", radix=2),
           Candidate(flow_id="local-fused-tile", processing_unit="radix2-scalar", radix=2),
           Candidate(flow_id="batch-folded", processing_unit="radix2-scalar", radix=2),
           Candidate(flow_id="baseline-global-stage", processing_unit="radix2-scalar", radix=2, block=100),
           Candidate(flow_id="baseline-global-stage", processing_unit="radix2-scalar", radix=2,
                     pipeline="double-buffer")]
    for c in bad:
        assert not check_lowering(c).legal, c
    m2b = Candidate(flow_id="local-fused-tile", processing_unit="dense-dot-fft64", radix=2, fused_tile=4096,
                    batch=64, batch_variant="spread", flow_realization="matrix-resident", ud=64)
    assert check_lowering(m2b).legal


def test_tail_groups_partition_is_complete():
    for tile, logn, glog, maxp in ((8, 10, 2, 4096), (64, 20, 3, 65536), (32, 16, 12, 1 << 24)):
        groups, singles = tail_groups(tile, logn, glog, maxp)
        covered = sorted([n0 << s for n0, g in groups for s in range(g)] + singles)
        assert covered == [1 << s for s in range(tile.bit_length() - 1, logn)]
        assert all((n0 << g) <= maxp and 2 <= g <= glog for n0, g in groups)


def test_local_matrix_decomposition_is_a_dft():
    n, tile = 256, 16
    rng = np.random.default_rng(0)
    x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
    from oracle.oracle import index_table

    br = index_table("bitrev", 8)
    state = (x[br].reshape(-1, tile) @ local_matrix(tile, "dit").T).reshape(n)
    # remaining DIT stages as plain radix-2 on the state
    for s in range(4, 8):
        h = 1 << s
        w = np.exp(-2j * np.pi * np.arange(h) / (2 * h))
        blk = state.reshape(-1, 2 * h)
        lo, hi = blk[:, :h], blk[:, h:] * w
        state = np.concatenate((lo + hi, lo - hi), axis=1).reshape(n)
    np.testing.assert_allclose(state, np.fft.fft(x), atol=1e-9)


def test_host_io_chunking_and_argument_checks():
    """Host-buffer execution: power-of-two chunk counts dividing the batch,
    ~64 MiB chunks; shape / dtype / device checks before anything runs."""
    import torch

    from bfft.entry import ExecutionPlan
    from bfft.host_io import default_chunks, execute_fft_plan_host

    def plan(n, b, tt="c2c"):
        return ExecutionPlan(n=n, batch=b, direction="dit", precision="fp32", selection_source="table", reason="t",
                             fallback=False, executed="fft_dit_matrix_batch" if b > 1 else "fft_dit_matrix",
                             block=256, params={"tile": min(n, 256)}, transform_type=tt,
                             transform_direction="inverse" if tt == "c2r" else "forward")
    assert default_chunks(plan(65536, 8192)) == 64     # 4 GiB -> 64 x 64 MiB
    assert default_chunks(plan(2048, 1)) == 1
    assert default_chunks(plan(1024, 48)) == 1        # 384 KiB: one chunk
    assert default_chunks(plan(1 << 20, 96)) == 8     # 768 MiB -> 12 wanted, largest power of two dividing 96 <= 12
    p = plan(1024, 16)
    with pytest.raises(TypeError):
        execute_fft_plan_host(p, torch.zeros(16, 1024, dtype=torch.complex128))
    with pytest.raises(ValueError):
        execute_fft_plan_host(p, torch.zeros(8, 1024, dtype=torch.complex64))
    with pytest.raises(TypeError):
        execute_fft_plan_host(p, [0.0])


def test_distributed_exchange_mode_validation():
    from bfft import dist as bdist

    class Stub:
        def empty(self, count):
            import torch
            return torch.empty(count, dtype=torch.complex64)

        def phase(self, k, x, out):
            out.copy_(x)

    f = bdist.DistributedFFT(256, n1=16, phases=Stub())
    assert f.exchange == "nccl"
    with pytest.raises(ValueError):
        bdist.DistributedFFT(256, n1=16, phases=Stub(), exchange="shm")


def test_composition_table_tamper_is_refused(tmp_path):
    import copy

    from bfft import composition

    t = composition.load_composition_table()
    if t is None:
        pytest.skip("no composition table promoted")
    bad = copy.deepcopy(t)
    bad["entries"][0]["candidate_ms"] *= 0.5
    path = tmp_path / "comp.json"
    path.write_text(json.dumps(bad))
    with pytest.raises(ConfigError):
        composition.load_composition_table(str(path))
