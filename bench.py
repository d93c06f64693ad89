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
    "sweep-2^12": {"n": 4096, "batch": 4096, "desc": "config 3 point: C2C forward N=4096, B=4096 (B*N=2^24)"},
    "sweep-2^20": {"n": 1 << 20, "batch": 16, "desc": "config 3 point: C2C forward N=2^20, B=16 (B*N=2^24)"},
}
SEED = 1234
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

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.gpu)], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
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
    threads = os.cpu_count() or 1
    # size one step to about 2 s of wall time so K+W steps stay within minutes
    probe = reference_cpu(wl["n"], 2.0, threads)
    rows = probe["rows"]
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(SEED)
    x = (rng.standard_normal((rows, wl["n"])) + 1j * rng.standard_normal((rows, wl["n"]))).astype(np.complex128)
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
    value = gflop(wl["n"], rows) * args.steps / t
    line = {
        "impl": "reference", "metric": "complex64 C2C FFT GFLOP/s (5N*log2N/t)", "value": value,
        "unit": "GFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "complex128 (reference CPU path is float64)",
        "data": f"synthetic iid N(0,1) re/im, seed {SEED}",
        "config": {"workload": wl["desc"], "n": wl["n"], "global_batch": wl["batch"],
                   "sample_rows_per_step": rows, "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": value, "unit": "GFLOP/s", "cores": probe["cores"], "kind": probe["kind"],
                         "sample": probe["sample"]},
        "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

def choose_plan(n: int, b: int):
    """The plan the public API resolves for this shape; when the table
    abstains (no B200 table bound to this environment) use the B200 batch
    local-fused core explicitly and say so."""
    from bfft import plan_fft
    from bfft.config import DeviceProfile
    from bfft.entry import ExecutionPlan

    p = plan_fft("dit", n, batch=b, profile_hash=DeviceProfile.load().hash())
    if not p.fallback:
        return p, "selector"
    log2n = n.bit_length() - 1
    tile = n if n <= 4096 else 1 << ((log2n + 1) // 2)
    return ExecutionPlan(n=n, batch=b, direction="dit", precision="fp32", selection_source="table",
                         reason="explicit B200 batch local-fused core (selector abstained: " + p.reason + ")",
                         fallback=False, executed="fft_dit_matrix_batch", block=256,
                         flow_id="local-fused-tile", flow_realization="matrix-resident",
                         processing_unit="dense-dot-fft64",
                         params={"tile": tile, "rows": 1, "variant": "spread", "batch": b}), "explicit"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("bfft", "reference"), default="bfft")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="5a")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]

    if args.impl == "reference":
        run_reference_arm(args, wl)
        return

    import torch
    import torch.distributed as dist

    import bfft
    from bfft import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and not (world == 1 and args.gpus == 1):
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            t = torch.ones(1, device=dev)
            dist.all_reduce(t)
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    n, btot = wl["n"], wl["batch"]
    if btot % world:
        raise SystemExit(f"batch {btot} does not split over {world} ranks")
    b = btot // world
    plan, plan_src = choose_plan(n, b)
    g = torch.Generator(device=dev).manual_seed(SEED + rank)
    x = torch.complex(torch.randn(b, n, device=dev, generator=g), torch.randn(b, n, device=dev, generator=g))
    torch.cuda.synchronize(dev)

    # ---- device-timed steps (inputs resident in HBM, 4 GiB > L2) ----
    for _ in range(args.warmup):
        y = bfft.execute_fft_plan(plan, x)
    del y
    from bfft.entry import native_plan_for

    native = native_plan_for(plan, local)
    stream = torch.cuda.current_stream(dev)
    barrier()
    l0 = _lib.launch_counter()
    with ClockSampler(local) as clk:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            y = bfft.execute_fft_plan(plan, x)
        end.record(stream)
        end.synchronize()
        barrier()
    launches = _lib.launch_counter() - l0
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    clocks = clk.summary()
    del y
    ms_step = elapsed_ms / args.steps
    value = gflop(n, btot) / (ms_step / 1e3)

    # ---- dominant kernel roofline: every launch of this flow is the
    # CTA-resident pass; each moves one read + one write of the shard ----
    peak, peak_src = measured_peaks()
    per_launch_ms = ms_step / max(native.launches, 1)
    bytes_per_launch = 16.0 * n * b
    achieved = bytes_per_launch / (per_launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "k_pass (CTA-resident Stockham pass)", "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_src,
                "traffic": None, "launches_per_step": native.launches,
                "algorithmic_bytes_per_launch": bytes_per_launch,
                "transform_hbm_gbs": 16.0 * n * b / (ms_step / 1e3) / 1e9}

    # ---- end to end through the public API with pinned host buffers ----
    e2e_steps = args.e2e_steps or max(1, min(args.steps, 5))
    xh = torch.empty((b, n), dtype=torch.complex64, pin_memory=True)
    xh.copy_(x)
    yh = torch.empty((b, n), dtype=torch.complex64, pin_memory=True)
    xd = torch.empty_like(x)
    del x
    for _ in range(1):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(bfft.execute_fft_plan(plan, xd), non_blocking=True)
    barrier()
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(e2e_steps):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(bfft.execute_fft_plan(plan, xd), non_blocking=True)
    e2.record(stream)
    e2.synchronize()
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2)) / e2e_steps
    e2e = {"value": gflop(n, btot) / (e2e_ms / 1e3), "unit": "GFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": int(xh.numel() * 8), "d2h_bytes_per_step": int(yh.numel() * 8),
           "path": "execute_fft_plan (bfft public API -> libbfft C ABI) with pinned host in/out"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = reference_cpu(n, 15.0, os.cpu_count() or 1)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        line = {
            "metric": "complex64 C2C FFT GFLOP/s (5N*log2N/t) and HBM GB/s vs roofline",
            "value": value, "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "complex64", "data": f"synthetic iid N(0,1) re/im, per-rank generator seed {SEED}+rank",
            "config": {"workload": wl["desc"], "n": n, "global_batch": btot, "per_rank_batch": b,
                       "parallelism": f"batch-shard x{world} (no data-path collective)",
                       "l2": "inputs larger than L2 (8 B * N * B per rank >= 512 MiB)",
                       "plan": plan.executed, "plan_params": plan.params, "plan_source": plan_src},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
