"""CUDA-graph capture of execute_fft_plan.

A plan executed once eagerly (which creates its native plan and caches) can
be captured into a CUDA graph and replayed: the multi-pass flows (whose
second and later passes are launched as programmatic dependents of the pass
before), the dedicated real flows and a single-pass flow.  Every replay must
equal the eager result bit for bit, also after the input buffer is refilled
between replays.
"""
import numpy as np
import pytest
import torch

from bfft import _lib
from bfft.entry import ExecutionPlan, execute_fft_plan

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _plan(executed, n, b, **kw):
    base = dict(n=n, batch=b, direction="dit", precision="fp32", selection_source="table", reason="t",
                fallback=False, executed=executed, block=256)
    base.update(kw)
    return ExecutionPlan(**base)


CASES = [
    ("c2c 2 passes", dict(executed="fft_dit_matrix_batch", n=65536, b=16, params={"tile": 256})),
    ("c2c 3 passes inverse", dict(executed="fft_dit_matrix_batch", n=1 << 20, b=4, params={"tile": 64},
                                  transform_direction="inverse", norm="ortho")),
    ("c2c 1 pass", dict(executed="fft_dit_matrix_batch", n=4096, b=32, params={"tile": 4096})),
    ("r2c", dict(executed="fft_dit_matrix_batch", n=65536, b=8, transform_type="r2c",
                 params={"tile": 256, "real_flow": "dedicated-r2c-pack-v1"})),
    ("c2r", dict(executed="fft_dit_matrix_batch", n=65536, b=8, transform_type="c2r",
                 transform_direction="inverse", params={"tile": 256, "real_flow": "dedicated-c2r-hermitian-v1"})),
]


def _input(p, g):
    if p.transform_type == "r2c":
        return torch.randn(p.batch, p.n, device=DEV, generator=g)
    cols = p.n // 2 + 1 if p.transform_type == "c2r" else p.n
    return torch.complex(torch.randn(p.batch, cols, device=DEV, generator=g),
                         torch.randn(p.batch, cols, device=DEV, generator=g))


@pytest.mark.parametrize("name, kw", CASES, ids=[c[0] for c in CASES])
def test_graph_replay_matches_eager(name, kw):
    kw = dict(kw)
    p = _plan(kw.pop("executed"), kw.pop("n"), kw.pop("b"), **kw)
    g = torch.Generator(device=DEV).manual_seed(7)
    x = _input(p, g)
    eager = execute_fft_plan(p, x).clone()  # creates the native plan and its caches

    side = torch.cuda.Stream(device=DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        execute_fft_plan(p, x)  # warm the side stream as torch's capture recipe asks
    torch.cuda.current_stream(DEV).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = execute_fft_plan(p, x)
    graph.replay()
    torch.cuda.synchronize(DEV)
    assert torch.equal(y, eager), name

    x2 = _input(p, g)
    eager2 = execute_fft_plan(p, x2).clone()
    x.copy_(x2)
    graph.replay()
    torch.cuda.synchronize(DEV)
    assert torch.equal(y, eager2), name
    ref = torch.fft.fft(x2.to(torch.complex128)) if p.transform_type == "c2c" and p.transform_direction == "forward" \
        else None
    if ref is not None:
        err = (torch.linalg.vector_norm(y.to(torch.complex128) - ref) / torch.linalg.vector_norm(ref)).item()
        assert err < 1e-6, (name, err)
    del graph
    assert _lib.device_status(0) == 0
