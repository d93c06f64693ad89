"""Reference parity at the BASELINE shapes, on row subsets.

``tests/golden/reference_rows.npz`` holds the reference's own output (its
Triton kernels run on the CPU, ``tests/golden/make_golden_rows.py``) for the
first rows of configurations 2, 3, 4 and 5a, at sampled positions; the inputs
are rebuilt from each case's seed.  For every case two B200 paths must match
the reference within 2e-6 relative L2 at those positions and float64 numpy
within 1e-6 per transform on the whole rows:

* the same runner (or dedicated real flow) with the same knobs as the
  reference used -- path parity;
* the plan bench.py times for that configuration's full shape (the selector's
  choice, or the explicit B200 plan when it abstains), executed on the rows.
"""
import json
import os

import numpy as np
import pytest
import torch

import bench
from bfft import runner
from bfft.entry import ExecutionPlan, execute_fft_plan
from bfft.error_metric import rel_l2, rel_l2_per_transform

from conftest import GOLDEN_DIR
from golden import row_cases

pytestmark = pytest.mark.gpu

TOL_REF = 2e-6
TOL_F64 = 1e-6
DEV = "cuda:0"

with open(os.path.join(GOLDEN_DIR, "reference_rows.json")) as _f:
    META = json.load(_f)["cases"]
LABELS = [c["label"] for c in row_cases.CASES if c["label"] in META]


@pytest.fixture(scope="module")
def rows():
    return np.load(os.path.join(GOLDEN_DIR, "reference_rows.npz"))


def _f64(case, x):
    if case["tt"] == "r2c":
        return np.fft.rfft(x.astype(np.float64), axis=-1)
    if case["tt"] == "c2r":
        return np.fft.irfft(x.astype(np.complex128), n=case["n"], axis=-1)
    x = x.astype(np.complex128)
    return np.fft.fft(x, axis=-1) if case["td"] == "forward" else np.fft.ifft(x, axis=-1)


def _same_path(case, t):
    b = case["rows"]
    if case["ref"] == "plan":
        p = ExecutionPlan(n=case["n"], batch=b, direction="dit", precision="fp32", selection_source="table",
                          reason="reference rows", fallback=False, executed=case["executed"], block=256,
                          params=dict(case["params"], batch=b), transform_type=case["tt"],
                          transform_direction=case["td"], norm="backward")
        return execute_fft_plan(p, t)
    return getattr(runner, case["ref"])(t, block=256, **case["knobs"])


def _product_path(case, t):
    plan, _ = bench.choose_plan(case["n"], case["full_batch"], case["tt"], case["td"])
    b = case["rows"]
    params = dict(plan.params or {})
    if "batch" in params:
        params["batch"] = b
    executed = plan.executed
    if b > 1 and executed in ("fft_dit_matrix", "fft_dif_matrix"):
        executed += "_batch"
    p = ExecutionPlan(**{**plan.__dict__, "batch": b, "params": params, "executed": executed})
    return execute_fft_plan(p, t), p


@pytest.mark.parametrize("label", LABELS)
def test_rows_match_the_reference(rows, label):
    case = next(c for c in row_cases.CASES if c["label"] == label)
    x = row_cases.case_input(case)
    t = torch.from_numpy(x).to(DEV)
    pos, want = rows[f"{label}__pos"], rows[f"{label}__out"]
    ref64 = _f64(case, x)
    for name, fn in (("same path", _same_path), ("product plan", lambda c, v: _product_path(c, v)[0])):
        y = fn(case, t)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert tuple(got.shape) == tuple(META[label]["out_shape"]), (label, name, got.shape)
        e_ref = rel_l2(got.reshape(-1)[pos], want)
        assert e_ref <= TOL_REF, (label, name, e_ref)
        e64 = rel_l2_per_transform(got, ref64)
        assert e64 <= TOL_F64, (label, name, e64)


def test_every_baseline_configuration_has_reference_rows():
    configs = {META[lab]["config"] for lab in LABELS}
    assert {"2", "3", "4", "5a"} <= configs
