"""Collected after every parity test (only the allocation-free entry point's
file comes later): no kernel of the GPU tests gave up a bounded wait (the TMA
pass records an expired mbarrier wait in the device status word)."""
import pytest

from bfft import _lib

pytestmark = pytest.mark.gpu


def test_no_bounded_wait_expired():
    assert _lib.device_status(0) == 0
