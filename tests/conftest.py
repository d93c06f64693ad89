"""Test configuration.

Two tiers, selected by marker (the reference splits host / ``hardware`` the
same way, pytest.ini:1-9):

* unmarked tests run anywhere (no GPU): the oracle against the reference's
  golden vectors, the host API, the C ABI's symbols and argument checks, and
  the multi-process logic on ``gloo`` CPU ranks;
* ``@pytest.mark.gpu`` tests need a B200: they call libbfft through the C ABI
  and compare with the oracle and the golden vectors.  They never skip when
  CUDA is missing -- run them with ``-m gpu`` on a GPU box.
"""
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "kunlunxin-fft_b200")
for p in (PKG_ROOT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_DIR = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(GOLDEN_DIR, "reference_vectors.npz"))


@pytest.fixture(scope="session")
def golden_meta():
    with open(os.path.join(GOLDEN_DIR, "reference_plans.json")) as f:
        return json.load(f)


def cplx(rng, shape):
    """iid N(0,1) real and imaginary parts, complex64 (the BASELINE inputs)."""
    return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)
