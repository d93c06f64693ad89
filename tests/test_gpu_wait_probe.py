"""Failure detection without a GPU fault: the kernels' bounded waits.

The TMA passes, the row-pair kernel and the fused single pass wait on
mbarriers (tile copies) and, in the fused pass, on dependency counters that
other CTAs publish.  Every such wait is bounded: when it runs out it sets a bit
of the device status word and the kernel returns, so a lost copy or a missing
publication shows up as an error the host reads, never as a hung GPU.

This test makes both kinds of wait run out on purpose -- an mbarrier that
nothing arrives on and a counter that nothing increments
(bfft_probe_bounded_waits) -- and checks that each reported its bit, that
clearing the word works, and that the same context then still computes a
correct transform.  No kernel traps, faults or spins without a limit.
"""
import numpy as np
import pytest
import torch

import bfft
from bfft import _lib
from oracle import oracle as O

from conftest import cplx

pytestmark = pytest.mark.gpu


def test_bounded_waits_expire_report_and_leave_the_context_usable():
    assert _lib.device_status(0) == 0, "a kernel reported an expired wait before the probe"
    L = _lib.load()
    stream = torch.cuda.current_stream(torch.device("cuda", 0))
    _lib.check(L.bfft_probe_bounded_waits(0, stream.cuda_stream), "bfft_probe_bounded_waits")
    status = _lib.device_status(0, clear=True)
    assert status & 1, f"the mbarrier wait did not report its expiry (status {status:#x})"
    assert status & 2, f"the dependency-counter wait did not report its expiry (status {status:#x})"
    assert _lib.device_status(0) == 0, "clearing the status word did not reset it"

    # the context is still healthy: a multi-pass and a fused transform, checked against float64
    rng = np.random.default_rng(2024)
    for n, b in ((4096, 8), (65536, 4)):
        x = cplx(rng, (b, n))
        y, rep = bfft.run_fft(torch.from_numpy(x).to("cuda:0"), "dit", profile_hash=None)
        torch.cuda.synchronize()
        assert O.rel_l2_rows(y.cpu().numpy(), O.fft_f64(x)) <= 1e-6, (n, b, rep.executed)
    assert _lib.device_status(0) == 0
