"""The measurement stage of the selector table builder on the device: a
small size matrix, timed and error-checked, builds into a table that loads
and selects under the live environment hash."""
import pytest

from bfft import table_builder as TB
from bfft.config import DeviceProfile
from bfft.envcheck import current_env_hash
from bfft.selector import select, validate_table

pytestmark = pytest.mark.gpu


def test_measure_and_build_small_matrix():
    shapes = [TB.Shape(256, 1, "dit"), TB.Shape(4096, 64, "dit"),
              TB.Shape(4096, 16, "dit", "c2r", "inverse", "backward", True)]
    run = TB.measure(shapes, sessions=2, trials=3, warmup=1)
    assert run["manifest"]["env_hash"] == current_env_hash()
    for rec in run["shapes"]:
        assert rec["extras_failed"] == [], rec["extras_failed"]
        for name, c in rec["candidates"].items():
            assert c["complete"] and c["median_ms"] > 0, name
            assert c["err_max"] < 1e-6, (rec["key"], name, c["err_max"])
    t = TB.build_table([run])
    assert validate_table(t) == []
    ph = DeviceProfile.load().hash()
    for e in t["entries"]:
        sel = select(e["direction"], e["N"], batch=e["batch"], profile_hash=ph, table=t,
                     transform_type=e.get("transform_type", "c2c"),
                     transform_direction=e.get("transform_direction", "forward"),
                     normalization=e.get("normalization", "backward"))
        assert sel.selected, sel.reason
    comp, notes = TB.build_composition_table([run], t)
    assert notes  # every c2c shape with 4-step candidates gets a verdict
    if comp is not None:
        from bfft.composition import table_violations

        assert table_violations(comp) == []
