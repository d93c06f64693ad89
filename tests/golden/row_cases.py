"""Row-subset golden cases at the BASELINE shapes the full golden set does not reach.

The reference is run (``make_golden_rows.py``) on the first rows of each
configuration -- rows of a batched FFT are independent, so a few rows of the
(B, N) job stand for all of them -- and its output is stored at a fixed set
of sampled positions.  The inputs are not stored: both the generator and the
GPU test rebuild them from the case's seed with ``case_input`` (numpy's PCG64
stream, identical on every box of this image), which keeps the fixture small.

Each case names the configuration it samples (``config``), the full shape of
that configuration (``full_batch``), the reference function that produced
the output (``ref``: a runner of ``src/xpu/runner.py`` or a dedicated real
flow through ``src/xpu/entry.py:execute_fft_plan``) and its knobs.
"""
from __future__ import annotations

import numpy as np

SAMPLES = 4096  # stored output positions per case (flattened over rows)

# config, transform, N, rows run, full batch of the config, reference function, knobs
CASES = [
    # config 2: batched C2C forward / inverse (1/N), all 64 rows
    dict(label="c2_fwd_1024x64", config="2", tt="c2c", td="forward", n=1024, rows=64, full_batch=64,
         ref="plan", executed="fft_dit_matrix_batch", params={"tile": 128, "rows": 8, "variant": "spread"}),
    dict(label="c2_inv_1024x64", config="2", tt="c2c", td="inverse", n=1024, rows=64, full_batch=64,
         ref="plan", executed="fft_dit_matrix_batch", params={"tile": 128, "rows": 8, "variant": "spread"}),
    dict(label="c2_fwd_2048x64", config="2", tt="c2c", td="forward", n=2048, rows=64, full_batch=64,
         ref="plan", executed="fft_dit_matrix_batch", params={"tile": 64, "rows": 8, "variant": "spread"}),
    dict(label="c2_inv_2048x64", config="2", tt="c2c", td="inverse", n=2048, rows=64, full_batch=64,
         ref="plan", executed="fft_dit_matrix_batch", params={"tile": 64, "rows": 8, "variant": "spread"}),
    # config 3: B*N = 2^24 sweep points beyond the golden set
    dict(label="c3_radix4_8192", config="3", tt="c2c", td="forward", n=1 << 13, rows=4, full_batch=1 << 11,
         ref="fft_dit_radix4_batch", knobs={}),
    dict(label="c3_matrix_8192", config="3", tt="c2c", td="forward", n=1 << 13, rows=4, full_batch=1 << 11,
         ref="fft_dit_matrix_batch", knobs={"tile": 64, "rows": 8}),
    dict(label="c3_radix4_2p17", config="3", tt="c2c", td="forward", n=1 << 17, rows=2, full_batch=1 << 7,
         ref="fft_dit_radix4_batch", knobs={}),
    dict(label="c3_matrix_2p17", config="3", tt="c2c", td="forward", n=1 << 17, rows=2, full_batch=1 << 7,
         ref="fft_dit_matrix_batch", knobs={"tile": 64, "rows": 8}),
    dict(label="c3_radix4_2p18", config="3", tt="c2c", td="forward", n=1 << 18, rows=2, full_batch=1 << 6,
         ref="fft_dit_radix4_batch", knobs={}),
    dict(label="c3_radix4_2p19", config="3", tt="c2c", td="forward", n=1 << 19, rows=2, full_batch=1 << 5,
         ref="fft_dit_radix4_batch", knobs={}),
    dict(label="c3_radix4_2p20", config="3", tt="c2c", td="forward", n=1 << 20, rows=2, full_batch=1 << 4,
         ref="fft_dit_radix4_batch", knobs={}),
    # config 5a rows (N = 65536 of B = 8192)
    dict(label="c5a_radix4_65536", config="5a", tt="c2c", td="forward", n=1 << 16, rows=4, full_batch=8192,
         ref="fft_dit_radix4_batch", knobs={}),
    # config 4: dedicated real flows (the reference's r2c / c2r table winner form)
    dict(label="c4_r2c_16384", config="4", tt="r2c", td="forward", n=1 << 14, rows=2, full_batch=256,
         ref="plan", executed="fft_dif_matrix_batch",
         params={"tile": 64, "rows": 8, "variant": "spread", "real_flow": "dedicated-r2c-pack-v1"}),
    dict(label="c4_c2r_16384", config="4", tt="c2r", td="inverse", n=1 << 14, rows=2, full_batch=256,
         ref="plan", executed="fft_dif_matrix_batch",
         params={"tile": 64, "rows": 8, "variant": "spread", "real_flow": "dedicated-c2r-hermitian-v1"}),
    dict(label="c4_r2c_65536", config="4", tt="r2c", td="forward", n=1 << 16, rows=2, full_batch=256,
         ref="plan", executed="fft_dif_matrix_batch",
         params={"tile": 64, "rows": 8, "variant": "spread", "real_flow": "dedicated-r2c-pack-v1"}),
    dict(label="c4_c2r_65536", config="4", tt="c2r", td="inverse", n=1 << 16, rows=2, full_batch=256,
         ref="plan", executed="fft_dif_matrix_batch",
         params={"tile": 64, "rows": 8, "variant": "spread", "real_flow": "dedicated-c2r-hermitian-v1"}),
]


def case_seed(label: str) -> int:
    """A fixed seed per case (stable across Python processes, unlike hash())."""
    return 20261202 + sum((i + 1) * ord(ch) for i, ch in enumerate(label))


def case_input(case: dict) -> np.ndarray:
    """The case's input rows: iid N(0,1) re/im complex64 (c2c), float32 (r2c),
    or the rfft of float32 N(0,1) rows cast to complex64 (c2r)."""
    rng = np.random.default_rng(case_seed(case["label"]))
    shape = (case["rows"], case["n"])
    if case["tt"] == "r2c":
        return rng.standard_normal(shape).astype(np.float32)
    if case["tt"] == "c2r":
        return np.fft.rfft(rng.standard_normal(shape).astype(np.float32).astype(np.float64)).astype(np.complex64)
    re = rng.standard_normal(shape).astype(np.float32)
    im = rng.standard_normal(shape).astype(np.float32)
    return (re + 1j * im).astype(np.complex64)


def sample_positions(case: dict, out_shape: tuple) -> np.ndarray:
    """Flattened output positions stored for the case (all of them when the
    output is smaller than SAMPLES)."""
    total = int(np.prod(out_shape))
    if total <= SAMPLES:
        return np.arange(total, dtype=np.int64)
    rng = np.random.default_rng(case_seed(case["label"]) + 1)
    return np.sort(rng.choice(total, size=SAMPLES, replace=False)).astype(np.int64)
