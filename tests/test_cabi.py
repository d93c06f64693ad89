"""The C ABI library (no GPU needed): it loads, exports exactly what
include/bfft.h declares, and rejects bad descriptors before touching CUDA."""
import ctypes
import os
import re

import pytest

from bfft import _build, _lib

HEADER = os.path.join(_build.INCLUDE, "bfft.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"BFFT_EXPORT\s+[\w\s\*]+?\b(bfft_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    _build.build(verbose=False)
    return _lib.load()


def test_library_is_built_for_sm100a(lib):
    meta = _build.build_meta()
    assert meta and meta["arch"] == "sm_100a" and "compute_100a" in " ".join(meta["flags"])
    assert meta["source_hash"] == _build.source_hash()


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.EXPORTS)


def test_api_version_and_counter(lib):
    assert lib.bfft_api_version() == 1
    assert _lib.launch_counter() >= 0
    assert isinstance(_lib.last_error(), str)


@pytest.mark.parametrize("field, value, exc", [
    ("runner", 99, ValueError), ("direction", 7, ValueError), ("n", 1000, ValueError),
    ("n", 0, ValueError), ("n", 1 << 31, ValueError), ("batch", 0, ValueError),
    ("block", 100, ValueError), ("tile", 48, ValueError), ("norm", 9, ValueError),
    ("transform_type", 5, ValueError), ("variant", 3, ValueError),
])
def test_plan_create_validates_before_cuda(lib, field, value, exc):
    d = _lib.make_desc("fft_dit", "dit", 1024, 1)
    setattr(d, field, value)
    with pytest.raises(exc):
        _lib.NativePlan(d)


def test_semantic_locks_and_spread_only(lib):
    d = _lib.make_desc("fft_dit", "dit", 64, 1, transform_type="r2c", transform_direction="inverse")
    with pytest.raises(ValueError, match="forward"):
        _lib.NativePlan(d)
    d = _lib.make_desc("fft_dit_matrix_batch", "dit", 64, 4, variant="folded")
    with pytest.raises(ValueError, match="spread"):
        _lib.NativePlan(d)
    d = _lib.make_desc("fft_dit", "dit", 2, 1, transform_type="r2c", real_flow=True)
    with pytest.raises(ValueError, match="N >= 4"):
        _lib.NativePlan(d)


def test_null_and_alias_arguments(lib):
    assert lib.bfft_execute(None, None, None, None, 0, None) == _lib.ERR_VALUE
    assert lib.bfft_bit_reverse_permute(ctypes.c_void_p(16), ctypes.c_void_p(16), 8, 1, 0, None) == _lib.ERR_VALUE
    assert lib.bfft_r2c_stitch(ctypes.c_void_p(16), ctypes.c_void_p(32), 2, 1, 1.0, 0, None) == _lib.ERR_SHAPE
    assert lib.bfft_index_map(3, 4, ctypes.c_void_p(16), 0, None) == _lib.ERR_VALUE
    assert lib.bfft_plan_destroy(None) == _lib.OK
