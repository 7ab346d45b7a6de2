#!/usr/bin/env python3
"""Benchmark of the B200 decode hot path: Q4_0 x Q8_1 mat-vec over the
Llama-3-8B layer shapes at batch 1, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step is one pass of the hot path over one batch of synthetic input: for each
of the four config-2 shapes (q/o 4096->4096, k/v 4096->1024, gate/up
4096->14336, down 14336->4096) quantise a fresh fp32 activation row to Q8_1
and multiply it by a Q4_0 weight matrix (8 kernel launches).  Successive steps
rotate over distinct weight copies totalling more than 3x the 126 MB L2, so
every step streams its weights from HBM.

value   = algorithmic bytes (weights + fp32 x + fp32 y, bin/mm-gbps.py:51-57)
          of all ranks / device time of the K steps (CUDA events, max over
          ranks), in GB/s.
e2e     = the same metric through the C-ABI with host buffers: each step
          copies its activations from pinned host memory, runs, copies y back
          and synchronises before the host reads it.
roofline: the gate/up mat-vec (4096 x 14336, the target shape) timed alone
          over back-to-back launches; achieved = its algorithmic bytes per
          launch / average launch time, against MEASURED_PEAKS.json hbm_gbs.
Multi-GPU (torchrun, one rank per GPU): weak scaling.  Each rank streams the
row shards of an N-times wider layer stack — the same per-GPU shapes — with
no collective on the data path (row-split mat-vecs exchange nothing).
--impl reference times the reference's own CPU path (prepare + evaluate per
row, oracle/_ref) on the host cores over a bounded sample of the same rows.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from p100_b200 import workloads as W  # noqa: E402

METRIC = "Q4_0 matvec HBM GB/s vs peak; batch-1 decode tok/s (8B/70B shapes) at 1/2/4/8 B200"
WORKLOAD = "Llama-3-8B layer shapes (q/o 4096x4096, k/v 4096x1024, gate/up 4096x14336, down 14336x4096), Q4_0 x Q8_1, batch 1"
SHAPES = [(name, k, rows) for name, k, rows in W.LLAMA3_8B_SHAPES]
TARGET = ("gate/up", 4096, 14336)
L2_BYTES = 126 * 1024 * 1024


def step_bytes():
    return sum(W.qmv_algorithmic_bytes(W.Q4_0, rows, k, 1) for _, k, rows in SHAPES)


def peak_gbs():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def ncu_traffic(name):
    """dram bytes per launch recorded from an ncu capture (profiles/<name>.md)."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ reference arm
def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path, on the host cores."""
    if rank != 0:
        return 0
    import oracle
    cores = oracle.host_cores()
    rows_per_shape = {"q/o": 32, "k/v": 32, "gate/up": 32, "down": 16}
    data = []
    for name, k, rows in SHAPES:
        n = rows_per_shape[name]
        data.append((name, k, n, W.weights(W.Q4_0, n, k, seed=k + rows), W.activations(1, k, seed=k)[0]))
    if oracle.Ref.available():
        ref, kind = oracle.Ref(), "reference"

        def one(qtype, w, n, k, x):
            return ref.evaluate_rows_threaded(qtype, w, n, k, x, cores)[1]
    else:
        orc, kind = oracle.oracle(), "port"

        def one(qtype, w, n, k, x):
            return orc.qmv_q81_threaded(qtype, w, n, k, orc.prepare(x), 1, cores)[1]
    nbytes = sum(n * (k // 32) * 18 + k * 4 + n * 4 for _, k, n, _, _ in data)
    for _ in range(args.warmup):
        for name, k, n, w, x in data:
            one(W.Q4_0, w, n, k, x)
    secs = 0.0
    for _ in range(args.steps):
        for name, k, n, w, x in data:
            secs += one(W.Q4_0, w, n, k, x)
    value = nbytes * args.steps / secs / 1e9
    sample = (f"{sum(rows_per_shape.values())} rows per step ({', '.join(f'{n} of {nm}' for nm, _, n, _, _ in data)}); "
              f"prepare + evaluate per row (evaluate also forms the exact and h16 paths)")
    if kind == "port":
        sample = sample.replace("prepare + evaluate per row (evaluate also forms the exact and h16 paths)",
                                "q81-only restatement of evaluate (oracle port)")
    line = {
        "metric": METRIC, "value": round(value, 6), "unit": "GB/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD + " (row sample)", "global_batch": 1, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(value, 6), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline_sample():
    """Reference CPU path on a bounded sample (rank 0, N=1): ~10 s of host work."""
    import oracle
    cores = oracle.host_cores()
    k, rows = TARGET[1], 96
    w = W.weights(W.Q4_0, rows, k, seed=3)
    x = W.activations(1, k, seed=4)[0]
    if oracle.Ref.available():
        ref, kind = oracle.Ref(), "reference"
        run = lambda: ref.evaluate_rows_threaded(W.Q4_0, w, rows, k, x, cores)[1]  # noqa: E731
    else:
        orc, kind = oracle.oracle(), "port"
        run = lambda: orc.qmv_q81_threaded(W.Q4_0, w, rows, k, orc.prepare(x), 1, cores)[1]  # noqa: E731
    run()
    secs, reps, t0 = 0.0, 0, time.time()
    while time.time() - t0 < 8.0 and reps < 400:
        secs += run()
        reps += 1
    nbytes = rows * (k // 32) * 18 + k * 4 + rows * 4
    return {"value": round(nbytes * reps / secs / 1e9, 6), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{rows} rows of the gate/up shape (k=4096), {reps} repetitions, prepare + evaluate per row"
            if kind == "reference" else f"{rows} rows of the gate/up shape, q81-only oracle port, {reps} repetitions"}


# ------------------------------------------------------------------ B200 arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

    import torch
    import p100_b200 as P

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    P.check(P.device_check(local))
    stream = torch.cuda.current_stream()

    # Weights: one host-generated set per shape, replicated on the device into
    # R copies so the steps rotate through more than 3x L2 of distinct bytes.
    per_copy = sum(W.weights(W.Q4_0, 1, k, 0).size * rows for _, k, rows in SHAPES)
    copies = max(4, int(np.ceil(3 * L2_BYTES / per_copy)) + 1)
    wdev = []
    for si, (name, k, rows) in enumerate(SHAPES):
        host = torch.from_numpy(W.weights(W.Q4_0, rows, k, seed=1000 + si + 17 * rank))
        base = host.cuda()
        wdev.append([base] + [base.clone() for _ in range(copies - 1)])
    xs = [torch.from_numpy(W.activations(1, k, seed=2000 + si)).cuda() for si, (_, k, _) in enumerate(SHAPES)]
    xqs = [torch.empty(P.q8_1_bytes(k, 1), dtype=torch.uint8, device="cuda") for _, k, _ in SHAPES]
    ys = [torch.empty(1, rows, dtype=torch.float32, device="cuda") for _, _, rows in SHAPES]
    launches_per_step = 2 * len(SHAPES)

    def step(i):
        c = i % copies
        for si, (name, k, rows) in enumerate(SHAPES):
            P.q8_1_quantize(xs[si], out=xqs[si], stream=stream)
            P.qmv(W.Q4_0, wdev[si][c], rows, k, xqs[si], 1, y=ys[si], stream=stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end))
    barrier()
    per_step = step_bytes()
    value = per_step * world * args.steps / (ms / 1e3) / 1e9

    # Per-shape device time (same rotation, each shape alone) and the target kernel.
    shape_gbs = {}
    target_ms = None
    reps = 8 * copies
    for si, (name, k, rows) in enumerate(SHAPES):
        P.q8_1_quantize(xs[si], out=xqs[si], stream=stream)
        for r in range(copies):
            P.qmv(W.Q4_0, wdev[si][r], rows, k, xqs[si], 1, y=ys[si], stream=stream)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for r in range(reps):
            P.qmv(W.Q4_0, wdev[si][r % copies], rows, k, xqs[si], 1, y=ys[si], stream=stream)
        e.record(stream)
        torch.cuda.synchronize()
        t = s.elapsed_time(e) / reps
        shape_gbs[f"{name} {k}x{rows}"] = {"us": round(t * 1e3, 3),
                                           "GB/s": round(W.qmv_algorithmic_bytes(W.Q4_0, rows, k, 1) / (t / 1e3) / 1e9, 1)}
        if (name, k, rows) == TARGET:
            target_ms = t

    # End to end through the C-ABI with host buffers.
    xh = [torch.from_numpy(W.activations(1, k, seed=3000 + si)).pin_memory() for si, (_, k, _) in enumerate(SHAPES)]
    yh = [torch.empty(1, rows, dtype=torch.float32).pin_memory() for _, _, rows in SHAPES]
    xd = [torch.empty(1, k, dtype=torch.float32, device="cuda") for _, k, _ in SHAPES]
    h2d = sum(t.numel() * 4 for t in xh)
    d2h = sum(t.numel() * 4 for t in yh)

    def e2e_step(i):
        c = i % copies
        for si, (name, k, rows) in enumerate(SHAPES):
            xd[si].copy_(xh[si], non_blocking=True)
            P.q8_1_quantize(xd[si], out=xqs[si], stream=stream)
            P.qmv(W.Q4_0, wdev[si][c], rows, k, xqs[si], 1, y=ys[si], stream=stream)
            yh[si].copy_(ys[si], non_blocking=True)
        stream.synchronize()   # the host reads this step's results

    for i in range(args.warmup):
        e2e_step(i)
    barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e))
    barrier()
    e2e_value = per_step * world * args.steps / (e2e_ms / 1e3) / 1e9
    P.check(P.device_error())

    peak, peak_kind = peak_gbs()
    target_bytes = W.qmv_algorithmic_bytes(W.Q4_0, TARGET[2], TARGET[1], 1)
    achieved = target_bytes / (target_ms / 1e3) / 1e9
    traffic = ncu_traffic("qmv_q4_0_4096x14336")
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": 1,
                   "parallelism": f"row-split shards x{world}, no data-path collective" if world > 1 else "1 GPU",
                   "l2": f"inputs larger than L2: {copies} rotating weight copies ({copies * per_copy / 1e6:.0f} MB)"},
        "roofline": {"bound": "hbm", "kernel": "qmv_bulk_kernel<Q4_0,1,1> gate/up 4096x14336",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic, "algorithmic_bytes": target_bytes, "us_per_launch": round(target_ms * 1e3, 3)},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "shapes": shape_gbs,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_sample()
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
