#!/usr/bin/env python
"""Benchmark of the batched C2C FFT hot path (BASELINE.json metric).

Default workload: config 5a -- batch-sharded complex64 C2C forward FFT,
N = 65536, B = 8192 (4 GiB) split over the ranks (one process per GPU, no
collective on the data path).  Metric: GFLOP/s = 5 N log2 N B / t over the
whole job (all ranks), t = max over ranks of the CUDA-event time of K steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl bfft|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

One JSON line on rank 0.  Besides the device-timed ``value`` it reports
``e2e`` (the same metric through the public API with pinned host buffers and
the H2D / D2H copies inside the timed region), ``roofline`` for the dominant
kernel, ``cpu_baseline`` (the reference's own C++ CPU FFT on this host's
cores, bounded sample), ``gpu_launches`` (libbfft launches in the timed
region) and ``clocks`` sampled by nvidia-smi during the timed region.
``--impl reference`` times the reference's CPU implementation instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "kunlunxin-fft_b200")
for _p in (PKG_ROOT, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

WORKLOADS = {
    "5a": {"n": 65536, "batch": 8192,
           "desc": "config 5a: batch-sharded C2C forward, N=65536, B=8192 (4 GiB complex64) split over ranks"},
    "sweep": {"n": 4096, "batch": 4096, "desc": "config 3 point: C2C forward, B*N=2^24 (set N with --n)"},
    "sweep-2^12": {"n": 4096, "batch": 4096, "desc": "config 3 point: C2C forward N=4096, B=4096 (B*N=2^24)"},
    "sweep-2^20": {"n": 1 << 20, "batch": 16, "desc": "config 3 point: C2C forward N=2^20, B=16 (B*N=2^24)"},
    "c1": {"n": 2048, "batch": 1, "desc": "config 1: single C2C forward FFT, N=2048, B=1 (rank-1)"},
    "c2-fwd": {"n": 2048, "batch": 64, "desc": "config 2: batched C2C forward, N=2048, B=64"},
    "c2-inv": {"n": 2048, "batch": 64, "td": "inverse",
               "desc": "config 2: batched C2C inverse (1/N), N=2048, B=64"},
    "c4-r2c": {"n": 65536, "batch": 256, "tt": "r2c",
               "desc": "config 4: R2C forward, N=65536, B=256 (float32 in, half spectrum out)"},
    "c4-c2r": {"n": 65536, "batch": 256, "tt": "c2r", "td": "inverse",
               "desc": "config 4: C2R inverse, N=65536, B=256 (half spectrum in, float32 out)"},
    "5b": {"n": 1 << 30, "batch": 1, "kind": "4step", "cpu_n": 1 << 20,
           "desc": "config 5b: one C2C forward of N=2^30 (8 GiB complex64); distributed 4-step over ranks (exchanges fused with the transposes, or NCCL all-to-all)"},
}
SEED = 1234
# One metric string for both arms (BASELINE.json's metric), so the two lines compare.
METRIC = "complex64 C2C FFT GFLOP/s (5N\u00b7log2N/t) and HBM GB/s vs roofline, 1-8 B200"
# DRAM bytes (read + write) per launch of the dominant kernel, from ncu
# captures of the same flow: config 5a from a 512-row case scaled by the rows
# processed; configs 3 and 4 captured at their full size.  Keyed by workload
# and transform length.
PROFILED_TRAFFIC = {
    ("5a", 65536): (10.21e9, "k_fused_fft<8,8>: 291.2 + 346.9 MB at B=512, scaled x16"),
    ("sweep", 2): (217.6e6, "k_rows_regs<1>"), ("sweep", 16): (215.2e6, "k_rows_shfl<4>"),
    ("sweep", 64): (217.7e6, "k_rows_shfl<6>"), ("sweep", 128): (215.0e6, "k_rows_shfl128"),
    ("sweep", 256): (214.0e6, "k_rows_pair<8>"), ("sweep", 1024): (214.2e6, "k_rows_pair<10>"),
    ("sweep", 4096): (215.9e6, "k_rows_pair<12>"), ("sweep", 8192): (279.3e6, "k_fused_fft<7,6>"),
    ("sweep", 32768): (289.8e6, "k_fused_fft<8,7>"), ("sweep", 131072): (287.4e6, "k_fused_fft<9,8>"),
    ("sweep", 1048576): (291.0e6, "k_fused_fft<10,10>"),
    ("c4-r2c", 65536): (111.1e6, "k_fused_fft<8,7> (the core)"), ("c4-c2r", 65536): (111.5e6, "k_fused_fft<8,7>"),
}
FALLBACK_HBM_GBS = 6650.0


def measured_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def gflop(n: int, rows: int) -> float:
    return 5.0 * n * math.log2(n) * rows / 1e9


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def _lines(self) -> int:
        try:
            with open(self.file.name) as f:
                return sum(1 for r in f if r.strip())
        except OSError:
            return 0

    def _wait_lines(self, n: int, limit_s: float) -> None:
        t0 = time.monotonic()
        while self._lines() < n and time.monotonic() - t0 < limit_s and self.proc.poll() is None:
            time.sleep(0.005)

    def __enter__(self):
        # The sampler is running (first sample written) before the timed
        # region starts; only samples after that point are summarised.
        self.skip = 0
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.gpu)], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
            self._wait_lines(1, 10.0)
            self.skip = self._lines()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self._wait_lines(self.skip + 2, 2.0)  # at least one sample at or after the region's end
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict | None:
        if self.proc is None or self.file is None:
            return None
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(", ") for r in f if r.strip()]
        os.unlink(self.file.name)
        rows = rows[max(self.skip - 1, 0):]  # the last sample before the region onwards
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU legs

def reference_cpu(n: int, target_s: float, threads: int) -> dict:
    """Time the reference's own C++ FFT (oracle/_ref, butterfly::fft_dit) on a
    bounded sample of rows; falls back to the C restatement if it is not built."""
    import numpy as np

    from oracle import oracle as O

    L = O.reference_lib()
    kind = "reference" if L is not None else "port"
    rng = np.random.default_rng(SEED)

    def run(rows, thr):
        x = (rng.standard_normal((rows, n)) + 1j * rng.standard_normal((rows, n))).astype(np.complex128)
        t0 = time.perf_counter()
        if L is not None:
            O.reference_fft_c128(x, dif=False, threads=thr)
        else:
            O.fft_f64(x)
        return time.perf_counter() - t0

    t1 = run(1, 1)
    thr = threads if L is not None else 1
    rows = max(thr, int(round(target_s * thr / max(t1, 1e-6))))
    rows = min(rows, 8192)
    rows = max(thr, (rows // thr) * thr)
    t = run(rows, thr)
    return {"value": gflop(n, rows) / t, "unit": "GFLOP/s", "cores": thr, "kind": kind,
            "sample": f"{rows} rows of N={n} (of the workload's batch), complex128, "
                      f"{'butterfly::fft_dit' if L is not None else 'C restatement'}; {t:.2f} s wall",
            "rows": rows, "seconds": t}


def run_reference_arm(args, wl) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # The reference's C++ FFT runs one transform per thread: a batched job
    # uses every host core, one 2^30-point transform (config 5b) runs on one
    # thread and is sampled at N = cpu_n (a full one takes minutes).
    threads = 1 if wl.get("kind") == "4step" else (os.cpu_count() or 1)
    n = wl.get("cpu_n", wl["n"])
    # size one step to about 2 s of wall time so K+W steps stay within minutes
    probe = reference_cpu(n, 2.0, threads)
    rows = probe["rows"]
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(SEED)
    x = (rng.standard_normal((rows, n)) + 1j * rng.standard_normal((rows, n))).astype(np.complex128)
    L = O.reference_lib()

    def step():
        if L is not None:
            O.reference_fft_c128(x, dif=False, threads=threads)
        else:
            O.fft_f64(x)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    t = time.perf_counter() - t0
    value = gflop(n, rows) * args.steps / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value,
        "unit": "GFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "complex128 (reference CPU path is float64)",
        "data": f"synthetic iid N(0,1) re/im, seed {SEED}",
        "config": {"workload": wl["desc"], "n": wl["n"], "global_batch": wl["batch"],
                   "sample_rows_per_step": rows, "sample_n": n, "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": value, "unit": "GFLOP/s", "cores": probe["cores"], "kind": probe["kind"],
                         "sample": probe["sample"]},
        "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

def choose_plan(n: int, b: int, tt: str = "c2c", td: str = "forward"):
    """The plan the public API resolves for this shape; when the table
    abstains (no B200 table bound to this environment, or a shape outside its
    matrix) use the B200 local-fused core explicitly and say so."""
    from bfft import plan_fft
    from bfft.config import DeviceProfile
    from bfft.entry import ExecutionPlan

    p = plan_fft("dit", n, batch=b, profile_hash=DeviceProfile.load().hash(), transform_type=tt,
                 transform_direction=td)
    if not p.fallback:
        return p, "selector"
    if tt != "c2c":
        real_flow = "dedicated-r2c-pack-v1" if tt == "r2c" else "dedicated-c2r-hermitian-v1"
        half = n // 2
        return ExecutionPlan(n=n, batch=b, direction="dit", precision="fp32", selection_source="table",
                             reason="explicit B200 dedicated real flow (selector abstained: " + p.reason + ")",
                             fallback=False, executed="fft_dit_matrix_batch" if b > 1 else "fft_dit_matrix",
                             block=256, flow_id=real_flow, flow_realization="matrix-resident",
                             processing_unit="dense-dot-fft64",
                             params={"tile": half if half <= 4096 or (half <= 65536 and b >= 2) else 256,
                                     "rows": 1, "variant": "spread", "batch": b, "real_flow": real_flow},
                             transform_type=tt, transform_direction=td), "explicit"
    # one CTA-resident pass up to 4096 points; 2^13..2^20 with a batch, the
    # fused single pass (tile = N); beyond, a 256-point local group and tail
    # passes of <= 2^9 points (every pass on the TMA-staged kernels); past 2^26
    # a 128-point local group (N = 2^30: 7 + 8 + 8 + 7 stages measured 1.5-2.5 %
    # faster than 8 + 8 + 7 + 7)
    tile = n if n <= 4096 or (n <= (1 << 20) and b >= 2) else (256 if n <= (1 << 26) else 128)
    executed = "fft_dit_matrix_batch" if b > 1 else "fft_dit_matrix"
    return ExecutionPlan(n=n, batch=b, direction="dit", precision="fp32", selection_source="table",
                         reason="explicit B200 local-fused core (selector abstained: " + p.reason + ")",
                         fallback=False, executed=executed, block=256,
                         flow_id="local-fused-tile", flow_realization="matrix-resident",
                         processing_unit="dense-dot-fft64",
                         params={"tile": tile, "rows": 1, "variant": "spread", "batch": b},
                         transform_direction=td), "explicit"


class Ctx:
    """Process-group plumbing shared by the workloads."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != args.gpus and not (self.world == 1 and args.gpus == 1):
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        if self.world > 1:
            t = self.torch.ones(1, device=self.dev)
            self.dist.all_reduce(t)
        self.torch.cuda.synchronize(self.dev)

    def gather(self, vals: list[float]) -> list[list[float]]:
        """Every rank's `vals` (same length on all ranks), rank order."""
        torch = self.torch
        t = torch.tensor(vals, dtype=torch.float64, device=self.dev)
        if self.world == 1:
            return [t.tolist()]
        out = torch.empty(self.world * len(vals), dtype=torch.float64, device=self.dev)
        self.dist.all_gather_into_tensor(out, t)
        return out.view(self.world, len(vals)).tolist()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn, steps: int, flush_l2: bool = False):
        """(max-over-ranks ms of `steps` calls of fn, launches, clocks).

        flush_l2: inputs smaller than L2 -- before every step a 256 MiB buffer
        is written (outside the timed spans) and only the call is timed; a
        device-side spin after the flush keeps the GPU busy while the host
        enqueues the call, so the span holds the device work, not the host's
        launch overhead."""
        from bfft import _lib

        torch = self.torch
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=self.dev) if flush_l2 else None
        self.barrier()
        l0 = _lib.launch_counter()
        with ClockSampler(self.local) as clk:
            if flush is None:
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record(self.stream)
                for _ in range(steps):
                    fn()
                end.record(self.stream)
                end.synchronize()
                ms = start.elapsed_time(end)
            else:
                spans = []
                for _ in range(steps):
                    flush.fill_(1)
                    torch.cuda._sleep(400_000)  # ~0.2 ms at B200 clocks, longer than one call's enqueue
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(self.stream)
                    fn()
                    b.record(self.stream)
                    spans.append((a, b))
                spans[-1][1].synchronize()
                ms = sum(a.elapsed_time(b) for a, b in spans)
            self.barrier()
        launches = _lib.launch_counter() - l0
        return self.max_over_ranks(ms), launches, clk.summary()

    def close(self):
        if self.world > 1:
            self.barrier()
            self.dist.destroy_process_group()


def _e2e(ctx, fn_dev, xh, yh, xd, steps):
    """Public-API call with pinned host in/out, copies inside the timed region."""
    torch = ctx.torch
    xd.copy_(xh, non_blocking=True)
    yh.copy_(fn_dev(xd), non_blocking=True)
    ctx.barrier()
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record(ctx.stream)
    for _ in range(steps):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(fn_dev(xd), non_blocking=True)
    e2.record(ctx.stream)
    e2.synchronize()
    ctx.barrier()
    return ctx.max_over_ranks(s2.elapsed_time(e2)) / steps


def _numa_node_of_gpu(ctx) -> int | None:
    """NUMA node the GPU hangs off (sysfs), None when not reported."""
    try:
        pr = ctx.torch.cuda.get_device_properties(ctx.dev)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            return int(f.read().strip())
    except (AttributeError, OSError, ValueError):
        return None


def _host_numa_nodes() -> int | None:
    """Online NUMA nodes of the host ("0-1" -> 2)."""
    try:
        with open("/sys/devices/system/node/online") as f:
            txt = f.read().strip()
        count = 0
        for part in txt.split(","):
            lo, _, hi = part.partition("-")
            count += int(hi or lo) - int(lo) + 1
        return count
    except (OSError, ValueError):
        return None


def link_rates(ctx, xh, yh) -> dict:
    """Host<->device copy rates of this step's pinned buffers, each direction
    alone (CUDA events, two copies each after one untimed), per rank, with
    where the GPUs and the host memory sit."""
    torch = ctx.torch
    xd = torch.empty(tuple(xh.shape), dtype=xh.dtype, device=ctx.dev)
    yd = torch.empty(tuple(yh.shape), dtype=yh.dtype, device=ctx.dev)
    rates = []
    for fn, nbytes in ((lambda: xd.copy_(xh, non_blocking=True), xh.numel() * xh.element_size()),
                       (lambda: yh.copy_(yd, non_blocking=True), yh.numel() * yh.element_size())):
        fn()
        ctx.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(ctx.stream)
        fn()
        fn()
        b.record(ctx.stream)
        b.synchronize()
        rates.append(nbytes / (a.elapsed_time(b) / 2 / 1e3) / 1e9)
        ctx.barrier()
    del xd, yd
    node = _numa_node_of_gpu(ctx)
    per = ctx.gather([rates[0], rates[1], -1.0 if node is None else float(node)])
    return {"h2d_gbs_per_rank": [round(r[0], 1) for r in per], "d2h_gbs_per_rank": [round(r[1], 1) for r in per],
            "gpu_numa_node_per_rank": [int(r[2]) if r[2] >= 0 else None for r in per],
            "host_numa_nodes": _host_numa_nodes(),
            "pinned_host_buffers": "torch pin_memory=True, first touched by each rank's process (no NUMA binding)",
            "how": "each direction alone: 2 full-buffer cudaMemcpyAsync per direction on the rank's stream, "
                   "CUDA events, all ranks at once"}


def api_wall(fn, trials: int) -> dict:
    """The reference's timing protocol (src/xpu/runner.py:1576-1635): warm-up,
    then interleaved trials of synchronised API wall time, with CUDA-event
    device time recorded beside it; median / p10 / p90."""
    from bfft import runner

    r = runner.time_call_detailed(fn, warmup=3, trials=trials, seed=0)
    return {"api_ms": r["api_ms"], "kernel_ms": r["kernel_ms"], "raw": r.get("raw"),
            "protocol": "bfft.runner.time_call_detailed: 3 warm-up calls, interleaved trials, "
                        "torch.cuda.synchronize() after each call; api_ms = host wall time of call + sync"}


def run_batch(args, wl, ctx) -> dict:
    """Configs 5a / 3: a batched C2C forward job, rows sharded over ranks."""
    import bfft
    from bfft import dist as bdist
    from bfft.entry import native_plan_for

    torch = ctx.torch
    n, btot = wl["n"], wl["batch"]
    tt, td = wl.get("tt", "c2c"), wl.get("td", "forward")
    first, b = bdist.batch_shard(btot, ctx.world, ctx.rank)
    plan, plan_src = choose_plan(n, b, tt, td)
    g = torch.Generator(device=ctx.dev).manual_seed(SEED + ctx.rank)
    if tt == "r2c":
        x = torch.randn(b, n, device=ctx.dev, generator=g)
    else:
        cols = n // 2 + 1 if tt == "c2r" else n
        x = torch.complex(torch.randn(b, cols, device=ctx.dev, generator=g),
                          torch.randn(b, cols, device=ctx.dev, generator=g))
    if b == 1:
        x = x[0].contiguous()
    # algorithmic bytes and flops of one step (real transforms: 2.5 N log2 N)
    in_row = 4 * n if tt == "r2c" else 8 * (n // 2 + 1) if tt == "c2r" else 8 * n
    out_row = 8 * (n // 2 + 1) if tt == "r2c" else 4 * n if tt == "c2r" else 8 * n
    flop_scale = 0.5 if tt != "c2c" else 1.0
    torch.cuda.synchronize(ctx.dev)
    for _ in range(args.warmup):
        y = bfft.execute_fft_plan(plan, x)
    del y
    native = native_plan_for(plan, ctx.local)
    small = in_row * b < (126 << 20)  # smaller than L2: flush between timed steps
    elapsed_ms, launches, clocks = ctx.timed(lambda: bfft.execute_fft_plan(plan, x), args.steps, flush_l2=small)
    ms_step = elapsed_ms / args.steps
    value = flop_scale * gflop(n, btot) / (ms_step / 1e3)

    # dominant kernel: every launch of this flow is the CTA-resident pass (or
    # the cluster kernel); each moves one read + one write of the shard (real
    # flows: the whole flow's algorithmic bytes over its launches)
    peak, peak_src = measured_peaks()
    per_launch_ms = ms_step / max(native.launches, 1)
    bytes_per_launch = float((in_row + out_row) * b) if tt != "c2c" else 16.0 * n * b
    achieved = bytes_per_launch / (per_launch_ms / 1e3) / 1e9
    traffic = PROFILED_TRAFFIC.get((args.workload, n))
    # per launch on this rank (b of the workload's rows), like `achieved`
    traffic_src = traffic[1] if traffic is not None and args.batch is None else None
    traffic = traffic[0] * b / wl["batch"] if traffic is not None and args.batch is None else None
    if native.launches == 1 and n > 4096 and tt == "c2c":
        kernel = "k_fused_fft (fused single pass)"
    elif native.launches == 1 and n in (256, 1024, 2048, 4096) and tt == "c2c":
        kernel = "k_rows_pair (warp-specialised paired row FFT)"
    else:
        kernel = "k_pass_tma / k_pass_tma_rows / k_rows_shfl (CTA-resident Stockham passes)"
    roofline = {"bound": "hbm", "kernel": kernel, "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_src,
                "traffic": traffic, "traffic_source": traffic_src, "launches_per_step": native.launches,
                "algorithmic_bytes_per_launch": bytes_per_launch,
                "transform_hbm_gbs": (in_row + out_row) * b / (ms_step / 1e3) / 1e9}

    # the reference's protocol: synchronised API wall time per call
    wall = api_wall(lambda: bfft.execute_fft_plan(plan, x), trials=args.api_trials)

    # end to end: host (pinned) in, host out, through the public host-buffer
    # entry; every step copies its input in and its result out
    from bfft.host_io import default_chunks, execute_fft_plan_host

    xh = torch.empty(tuple(x.shape), dtype=x.dtype, pin_memory=True)
    xh.copy_(x)
    oshape = (*x.shape[:-1], n // 2 + 1 if tt == "r2c" else n)
    yh = torch.empty(oshape, dtype=torch.float32 if tt == "c2r" else torch.complex64, pin_memory=True)
    del x
    chunks = default_chunks(plan)
    steps = args.e2e_steps or max(1, min(args.steps, 5))
    execute_fft_plan_host(plan, xh, yh, chunks=chunks)
    ctx.barrier()
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record(ctx.stream)
    for _ in range(steps):
        execute_fft_plan_host(plan, xh, yh, chunks=chunks)
    e2.record(ctx.stream)
    e2.synchronize()
    ctx.barrier()
    e2e_ms = ctx.max_over_ranks(s2.elapsed_time(e2)) / steps
    e2e = {"value": flop_scale * gflop(n, btot) / (e2e_ms / 1e3), "unit": "GFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": int(xh.numel() * xh.element_size()) * ctx.world,
           "d2h_bytes_per_step": int(yh.numel() * yh.element_size()) * ctx.world,
           "chunks": chunks,
           "path": "execute_fft_plan_host (bfft public API -> libbfft bfft_stream_execute): pinned host in/out, "
                   "batch in chunks, copy in / transform / copy out overlapped on three streams",
           "host_links": link_rates(ctx, xh, yh)}
    return {"value": value, "ms_step": ms_step, "launches": launches, "clocks": clocks, "roofline": roofline,
            "e2e": e2e, "scaling": "strong", "api_wall": wall,
            "config": {"workload": wl["desc"], "n": n, "global_batch": btot, "per_rank_batch": b,
                       "transform": f"{tt}/{td}", "flop_convention": "5 N log2 N" if tt == "c2c" else "2.5 N log2 N",
                       "parallelism": f"batch-shard x{ctx.world} (no data-path collective)",
                       "l2": ("inputs larger than L2" if not small
                              else "input smaller than L2: a 256 MiB buffer is written before every step, "
                                   "only the call is timed"),
                       "plan": plan.executed, "plan_params": plan.params, "plan_source": plan_src},
            "gflop_per_step": gflop(n, btot)}


def run_4step(args, wl, ctx) -> dict:
    """Config 5b: one transform of N = 2^30.  One GPU: three CTA-resident
    passes of 2^10; P GPUs: the slab-distributed 4-step with NCCL
    all-to-alls (bfft.dist.DistributedFFT)."""
    import bfft
    from bfft import dist as bdist
    from bfft.entry import native_plan_for

    torch = ctx.torch
    n = wl["n"]
    slab = n // ctx.world
    g = torch.Generator(device=ctx.dev).manual_seed(SEED + ctx.rank)
    x = torch.complex(torch.randn(slab, device=ctx.dev, generator=g), torch.randn(slab, device=ctx.dev, generator=g))
    peak, peak_src = measured_peaks()
    if ctx.world == 1:
        plan, plan_src = choose_plan(n, 1)
        fn = lambda t: bfft.execute_fft_plan(plan, t)  # noqa: E731
        desc = {"plan": plan.executed, "plan_params": plan.params, "plan_source": plan_src,
                "parallelism": "1 GPU"}
    else:
        f = bdist.DistributedFFT(n, device=ctx.dev, exchange=args.exchange)
        fn = f.execute
        how = ("transposes fused with the exchanges: peer stores over NVLink into the other ranks' buffers "
               "(CUDA IPC), stream-ordered barriers" if f.exchange == "p2p" else "NCCL all_to_all_single x3")
        desc = {"plan": f"DistributedFFT (4-step, {how})", "exchange": f.exchange, "factors": [f.n1, f.n2],
                "parallelism": f"slab x{ctx.world}, 3 exchanges per transform"}
    for _ in range(args.warmup):
        y = fn(x)
    del y
    elapsed_ms, launches, clocks = ctx.timed(lambda: fn(x), args.steps)
    ms_step = elapsed_ms / args.steps
    value = gflop(n, 1) / (ms_step / 1e3)
    if ctx.world == 1:
        native = native_plan_for(plan, ctx.local)
        per_launch_ms = ms_step / max(native.launches, 1)
        bpl = 16.0 * n
        roofline = {"bound": "hbm", "kernel": "k_pass_tma (TMA column pass; CTA-resident Stockham)",
                    "achieved": bpl / (per_launch_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                    "peak_source": peak_src, "traffic": None, "launches_per_step": native.launches,
                    "algorithmic_bytes_per_launch": bpl, "transform_hbm_gbs": 16.0 * n / (ms_step / 1e3) / 1e9}
    else:
        # the exchanges bound this path: 3 all-to-alls, each sending (P-1)/P
        # of the rank's slab over NVLink
        wire = 3.0 * 8.0 * slab * (ctx.world - 1) / ctx.world
        nvl = wire / (ms_step / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "whole step (transposes with exchanges, row passes)",
                    "achieved": 16.0 * slab / (ms_step / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                    "peak_source": peak_src, "traffic": None,
                    "nvlink": {"bytes_per_step_per_gpu": wire, "achieved_gbs_per_direction": nvl,
                               "peak_gbs_per_direction": 770.0, "frac": nvl / 770.0,
                               "peak_source": "measured peer copy on this pool (recipe figure)"}}
    roofline["frac"] = roofline["achieved"] / peak

    xh = torch.empty(slab, dtype=torch.complex64, pin_memory=True)
    xh.copy_(x)
    yh = torch.empty(slab, dtype=torch.complex64, pin_memory=True)
    xd = torch.empty_like(x)
    del x
    e2e_ms = _e2e(ctx, fn, xh, yh, xd, args.e2e_steps or 2)
    e2e = {"value": gflop(n, 1) / (e2e_ms / 1e3), "unit": "GFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": 8 * n, "d2h_bytes_per_step": 8 * n,
           "path": ("execute_fft_plan" if ctx.world == 1 else "DistributedFFT.execute") +
                   " with pinned host slabs in/out"}
    return {"value": value, "ms_step": ms_step, "launches": launches, "clocks": clocks, "roofline": roofline,
            "e2e": e2e, "scaling": "strong",
            "config": {"workload": wl["desc"], "n": n, "global_batch": 1,
                       "l2": "input 8 GiB, larger than L2", **desc},
            "gflop_per_step": gflop(n, 1)}


def secondary_5b(args, ctx) -> dict:
    """Config 5b beside the 5a headline, so every scaling run records it: one
    C2C forward of N = 2^30 (the single-GPU four-pass plan on one GPU, the
    slab-distributed 4-step of bfft.dist.DistributedFFT over the ranks
    otherwise), timed like the headline (max over ranks of CUDA-event time),
    and the same path checked at N = 2^24 against float64 numpy.fft on
    rank 0 (the slabs gathered there)."""
    import numpy as np

    import bfft
    from bfft import dist as bdist

    torch = ctx.torch
    res = {"workload": "config 5b: one C2C forward of N=2^30 (8 GiB complex64), slab per rank",
           "exchange": None}

    def make(n, order="natural"):
        if ctx.world == 1:
            plan, _ = choose_plan(n, 1)
            return (lambda t: bfft.execute_fft_plan(plan, t)), None, f"{plan.executed} tile {plan.params['tile']}"
        f = bdist.DistributedFFT(n, device=ctx.dev, exchange=args.exchange, output_order=order)
        res["exchange"] = f.exchange
        return f.execute, f, f"DistributedFFT {f.n1}x{f.n2}, {f.exchange} exchanges, {order} output"

    def parity(order):
        """rel L2 at N = 2^24 against float64 numpy.fft (rank 0; None elsewhere)."""
        nc = 1 << 24
        g = torch.Generator(device=ctx.dev).manual_seed(SEED + 77 + ctx.rank)
        xc = torch.complex(torch.randn(nc // ctx.world, device=ctx.dev, generator=g),
                           torch.randn(nc // ctx.world, device=ctx.dev, generator=g))
        fn, obj, _ = make(nc, order)
        yc = fn(xc)
        parts = []
        for t in (xc, yc):
            flat = torch.view_as_real(t).reshape(-1).contiguous()
            if ctx.world > 1:
                full = torch.empty(flat.numel() * ctx.world, dtype=flat.dtype, device=ctx.dev)
                ctx.dist.all_gather_into_tensor(full, flat)
            else:
                full = flat
            parts.append(full)
        rel = None
        if ctx.rank == 0:
            xa = parts[0].view(-1, 2).cpu().numpy().astype(np.float64)
            ya = parts[1].view(-1, 2).cpu().numpy().astype(np.float64)
            ref = np.fft.fft(xa[:, 0] + 1j * xa[:, 1])
            if order == "transposed":  # rank blocks of whole columns k1, one after another
                ref = ref.reshape(obj.n2, obj.n1).T.reshape(-1)
            got = ya[:, 0] + 1j * ya[:, 1]
            rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        del xc, yc, parts, fn, obj
        ctx.barrier()
        return nc, rel

    def timed(order):
        n = 1 << 30
        slab = n // ctx.world
        g = torch.Generator(device=ctx.dev).manual_seed(SEED + ctx.rank)
        x = torch.complex(torch.randn(slab, device=ctx.dev, generator=g),
                          torch.randn(slab, device=ctx.dev, generator=g))
        fn, obj, path = make(n, order)
        for _ in range(3):
            y = fn(x)
        del y
        ms, launches, clocks = ctx.timed(lambda: fn(x), args.steps_5b)
        ms /= args.steps_5b
        out = {"path": path, "n": n, "ms_per_step": ms, "steps": args.steps_5b, "warmup": 3,
               "gflops": gflop(n, 1) / (ms / 1e3), "gpu_launches": int(launches),
               "transform_hbm_gbs_per_gpu": 16.0 * slab / (ms / 1e3) / 1e9, "clocks": clocks}
        if obj is not None:
            # one more (untimed) execution with events between the steps: where the time goes
            trace = []
            obj.execute(x, trace=trace)
            torch.cuda.synchronize(ctx.dev)
            steps = {}
            for (_, e0), (name, e1) in zip(trace, trace[1:]):
                steps.setdefault(name, []).append(round(e0.elapsed_time(e1), 3))
            out["step_ms_rank"] = {"rank": ctx.rank, "steps": steps}
            ctx.barrier()
        if ctx.world > 1:
            wire = (3.0 if order == "natural" else 2.0) * 8.0 * slab * (ctx.world - 1) / ctx.world
            out["nvlink"] = {"bytes_per_step_per_gpu": wire, "gbs_per_direction": wire / (ms / 1e3) / 1e9,
                             "peak_gbs_per_direction": 770.0, "peak_source": "measured peer copy on this pool"}
        del x, fn, obj
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
        return out

    nc, rel = parity("natural")
    res.update(timed("natural"))
    res.update({"parity_n": nc, "rel_l2_vs_float64": rel})
    if ctx.world > 1:
        # the explicit transposed-output mode: two exchanges, rank r keeps
        # columns k1 in [r N1/P, (r+1) N1/P) of the N1 x N2 output view
        nc, rel_t = parity("transposed")
        t = timed("transposed")
        t.update({"parity_n": nc, "rel_l2_vs_float64": rel_t,
                  "layout": "rank r holds out[k1'][k2] = X[k2 N1 + r N1/P + k1']"})
        res["transposed_output"] = t
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("bfft", "reference"), default="bfft")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="5a")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--api-trials", type=int, default=20,
                    help="trials of the reference-style synchronised API wall-time protocol")
    ap.add_argument("--steps-5b", type=int, default=5, help="timed steps of the config-5b secondary line")
    ap.add_argument("--no-5b", action="store_true", help="skip the config-5b secondary measurement (5a only)")
    ap.add_argument("--rows-out", default=None,
                    help="write the raw rows (API wall / device time of every trial, the JSON line) to this file")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=("p2p", "nccl"), default=None,
                    help="5b on 2+ GPUs: fused peer-store exchanges (default) or NCCL all-to-alls")
    ap.add_argument("--n", type=int, default=None,
                    help="sweep workload: transform length N (power of two <= 2^24), batch 2^24 / N")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch: a small case of the same kernels for profiler captures "
                         "(the line is marked profile_case and is not a bench figure)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = dict(WORKLOADS[args.workload])
    if args.n is not None:
        if args.workload != "sweep" or args.n < 2 or args.n & (args.n - 1) or args.n > (1 << 24):
            raise SystemExit("--n needs --workload sweep and a power of two in [2, 2^24]")
        wl.update(n=args.n, batch=(1 << 24) // args.n,
                  desc=f"config 3 point: C2C forward N={args.n}, B={(1 << 24) // args.n} (B*N=2^24)")
    if args.batch is not None:
        wl.update(batch=int(args.batch), desc=wl["desc"] + f" [profile case: batch {args.batch}]", profile_case=True)

    if args.impl == "reference":
        run_reference_arm(args, wl)
        return

    ctx = Ctx(args)
    res = run_4step(args, wl, ctx) if wl.get("kind") == "4step" else run_batch(args, wl, ctx)
    sec = None
    if args.workload == "5a" and args.batch is None and not args.no_5b:
        try:
            sec = secondary_5b(args, ctx)
        except Exception as e:  # noqa: BLE001 - the headline line is printed regardless; the error is reported
            sec = {"workload": "config 5b", "error": f"{type(e).__name__}: {e}"[:300]}

    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        cpu_n = wl.get("cpu_n", wl["n"])
        cpu = reference_cpu(cpu_n, 15.0, 1 if wl.get("kind") == "4step" else (os.cpu_count() or 1))
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if ctx.rank == 0:
        line = {
            "metric": METRIC,
            "value": res["value"], "unit": "GFLOP/s", "n_gpus": ctx.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_step"], "higher_is_better": True,
            "scaling": res["scaling"], "vs_baseline": None, "dtype": "complex64",
            "data": f"synthetic iid N(0,1) re/im, per-rank generator seed {SEED}+rank",
            "config": res["config"], "roofline": res["roofline"], "cpu_baseline": cpu, "e2e": res["e2e"],
            "gpu_launches": int(res["launches"]), "clocks": res["clocks"],
        }
        if res.get("api_wall") is not None:
            line["api_wall"] = res["api_wall"]
        if sec is not None:
            line["secondary_5b"] = sec
        if wl.get("profile_case"):
            line["profile_case"] = True
        raw = (line.get("api_wall") or {}).pop("raw", None)
        if args.rows_out:
            with open(args.rows_out, "w") as f:
                json.dump({"line": line, "api_wall_trials": raw}, f, indent=1)
        print(json.dumps(line), flush=True)
    ctx.close()


if __name__ == "__main__":
    main()
