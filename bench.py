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

value   = algorithmic bytes of the step (weights + fp32 x + fp32 y,
          bin/mm-gbps.py:51-57) / device time (CUDA events, max over ranks),
          in GB/s: the median over interleaved rounds of K steps each, the
          rounds repeated until they span at least a second (`rounds`).
          N = 1: the whole step on one GPU.  N > 1 (torchrun, one rank per
          GPU): the same layer step split over the ranks, strong scaling —
          q/o and down along k (partial sums, each all-reduced with
          p100_tp_allreduce_sum inside the timed region: one kernel over NVLink
          peer memory where the GPUs reach each other, else NCCL), k/v and
          gate/up by rows; `replicated` keeps the
          weak-scaling figure (every rank the whole shapes, no collective).
e2e     = the headline's step through the C-ABI with host buffers: each step
          copies its activations from pinned host memory, runs, copies y back
          and synchronises before the host reads it.
roofline: the gate/up mat-vec (4096 x 14336, the target shape) timed alone
          over back-to-back launches in every round; achieved = its
          algorithmic bytes per launch / median launch time, against
          MEASURED_PEAKS.json hbm_gbs.
--impl reference times the reference's own CPU path (prepare + evaluate per
row, oracle/_ref) on the host cores over a bounded sample of the same rows.
decode  = configs 4/5: batch-1 decode tokens/s of the Llama-3 8B and 70B
          shapes (random-init Q4_0, KV prefilled to 4096 / 8192), split over
          the ranks (TP = N), with each GPU's bytes per token against the HBM
          roofline; at N > 1 the 8B model's tp_parity against the unsplit
          model and the exchange's cost per layer, and `collective`
          (p100_tp_allreduce_sum and ncclAllReduce latency and bus bandwidth
          at the exchange sizes).
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
    """nvidia-smi clocks and throttle reasons sampled during the timed region
    (every 20 ms; the sampler's first line is awaited before timing starts).
    A timed region shorter than the interval may hold no sample: the summary
    then uses the samples just around it and says so."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []
        self.first = self.last = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            deadline = time.time() + 5.0
            while not self.lines and time.time() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.first = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.last = len(self.lines)
        if self.proc:
            time.sleep(0.05)   # one more sample just after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        window, where = self.lines[self.first:self.last], "during the timed region"
        if not window:
            window = self.lines[max(0, self.first - 2):self.first + 2]
            where = "just before and after the timed region (shorter than the 20 ms interval)"
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in window:
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
            return {"error": (self.lines[:2] or ["nvidia-smi gave no samples"])[0][:200]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "window": where}


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
def capture(torch, fn):
    """A CUDA graph of fn()'s stream work (the C-ABI calls it makes), captured
    after one eager call has configured every kernel."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        fn()
    return g


def time_graphs(torch, graphs, n, stream):
    """Device ms of n replays cycling through graphs (events on the stream)."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(n):
        graphs[i % len(graphs)].replay()
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e)


FA_CONTEXTS = (512, 4096, 16384, 32768)


def h16_section(torch, P, stream):
    """The h16 activation path (qmv::h16_model; HFMA2 chain 16) on the
    Llama-3-8B layer shapes at batch 1, Q4_0: graph-replayed back-to-back
    calls over rotating weight copies beyond 3x L2.  GB/s counts the weights,
    the fp16 activations with their {scale, sum} record, and the outputs."""
    peak = peak_gbs()[0]
    out = {}
    for si, (name, k, rows) in enumerate(SHAPES):
        base = torch.from_numpy(W.weights(W.Q4_0, rows, k, seed=6000 + si)).cuda()
        copies = max(4, int(np.ceil(3 * L2_BYTES / base.numel())) + 1)
        ws = [base] + [base.clone() for _ in range(copies - 1)]
        h, ss = P.h16_prepare(torch.from_numpy(W.activations(1, k, seed=6100 + si)).cuda())
        y = torch.empty(1, rows, dtype=torch.float32, device="cuda")
        n_in_graph = max(16, copies)
        g = capture(torch, lambda: [P.qmv_h16(W.Q4_0, ws[r % copies], rows, k, h, ss, 1, 16, y=y)
                                    for r in range(n_in_graph)])
        time_graphs(torch, [g], 2, stream)
        reps = 5
        us = time_graphs(torch, [g], reps, stream) / (reps * n_in_graph) * 1e3
        nbytes = base.numel() + k * 2 + (k // 32) * 8 + rows * 4
        out[f"{name} {k}x{rows}"] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                                     "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
        del g, ws, base
    return out


def fa_section(torch, P, stream):
    """Config 3: FA-vec decode, 32 query / 8 KV heads, d 128, per context
    length; K/V rotate over copies totalling more than 3x L2; a CUDA graph of
    back-to-back calls, CUDA events around its replays."""
    out = {}
    peak, _ = peak_gbs()
    for seq in FA_CONTEXTS:
        q, k, v = W.attention_inputs(1, 32, 8, seq, 128, seed=seq)
        copies = max(2, int(np.ceil(3 * L2_BYTES / (k.nbytes * 2))) + 1)
        qd = torch.from_numpy(q).cuda()
        kd = [torch.from_numpy(k).cuda() for _ in range(copies)]
        vd = [torch.from_numpy(v).cuda() for _ in range(copies)]
        desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=seq)
        ws = P.fa_workspace(desc)
        o = torch.empty(1, 32, 1, 128, device="cuda")
        lse = torch.empty(1, 32, 1, device="cuda")
        reps = max(4, 64 // copies)
        g = capture(torch, lambda: [P.fa_decode(desc, qd, kd[r % copies], vd[r % copies], o=o, lse=lse, ws=ws)
                                    for r in range(copies * reps)])
        time_graphs(torch, [g], 2, stream)
        n = 10
        us = time_graphs(torch, [g], n, stream) / (n * copies * reps) * 1e3
        nbytes = W.fa_algorithmic_bytes(1, 32, 8, seq, 128)
        out[str(seq)] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                         "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
        del kd, vd
    return out


def kv_quant_section(torch, P, stream):
    """Quantised K/V cache (llama.cpp -ctk/-ctv q8_0, q4_0; bench/phase0.sh:127):
    (1) FA-vec decode over q8_0 / q4_0 K/V, config 3's heads (32 q / 8 kv,
    d 128) per context length, timed as fa_section times fp16; GB/s counts the
    quantised K/V bytes.  (2) p100_kv_to_f16 on the reference's conversion
    shapes (bench/micro/dequant_nc.cu:209-214; its token-major view), GB/s =
    block bytes read + fp16 bytes written, sources rotating beyond 3x L2."""
    peak = peak_gbs()[0]
    fa, conv = {}, {}
    for kv_type, name in ((P.KV_Q8_0, "q8_0"), (P.KV_Q4_0, "q4_0")):
        fa[name] = {}
        for seq in FA_CONTEXTS:
            q, _, _ = W.attention_inputs(1, 32, 8, seq, 128, seed=seq)
            kb = W.kv_cache_blocks(kv_type, 1, 8, seq, 128, seed=seq + 1)
            vb = W.kv_cache_blocks(kv_type, 1, 8, seq, 128, seed=seq + 2)
            copies = max(2, int(np.ceil(3 * L2_BYTES / (kb.nbytes * 2))) + 1)
            qd = torch.from_numpy(q).cuda()
            kd = [torch.from_numpy(kb).cuda() for _ in range(copies)]
            vd = [torch.from_numpy(vb).cuda() for _ in range(copies)]
            desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=seq, kv_type=kv_type)
            ws = P.fa_workspace(desc)
            o = torch.empty(1, 32, 1, 128, device="cuda")
            lse = torch.empty(1, 32, 1, device="cuda")
            reps = max(4, 64 // copies)
            g = capture(torch, lambda: [P.fa_decode(desc, qd, kd[r % copies], vd[r % copies], o=o, lse=lse, ws=ws)
                                        for r in range(copies * reps)])
            time_graphs(torch, [g], 2, stream)
            n = 10
            us = time_graphs(torch, [g], n, stream) / (n * copies * reps) * 1e3
            nbytes = W.fa_algorithmic_bytes(1, 32, 8, seq, 128, kv_type)
            fa[name][str(seq)] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                                  "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
            del kd, vd, g
        conv[name] = {}
        for d, n_kv, nh in ((64, 7680, 8), (128, 16384, 8), (256, 16384, 2), (256, 32768, 4)):
            nb = d // 32
            bb = P.KV_BLOCK_BYTES[kv_type]
            src_bytes = nb * nh * n_kv * bb
            copies = max(2, int(np.ceil(3 * L2_BYTES / (src_bytes + n_kv * nh * d * 2))) + 1)
            srcs = [torch.randint(0, 256, (src_bytes,), dtype=torch.uint8, device="cuda") for _ in range(copies)]
            for s_ in srcs:   # finite fp16 scales: d in [0.01, 0.02)
                s_.view(-1, bb)[:, 1] = 0x20 + (s_.view(-1, bb)[:, 1] & 3)
            dst = torch.empty(nh, n_kv, d, dtype=torch.float16, device="cuda")
            args = (d, n_kv, nh, 1, nb * nh, nb, nb * nh * n_kv)
            reps = max(8, 64 // copies)
            g = capture(torch, lambda: [P.kv_to_f16(kv_type, srcs[r % copies], *args, out=dst)
                                        for r in range(copies * reps)])
            time_graphs(torch, [g], 2, stream)
            n = 10
            us = time_graphs(torch, [g], n, stream) / (n * copies * reps) * 1e3
            nbytes = src_bytes + n_kv * nh * d * 2
            conv[name][f"d{d}_kv{n_kv}_h{nh}"] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                                                  "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
            del srcs, g
    return {"fa_decode": fa, "kv_to_f16": conv}


DECODE_MODELS = {   # BASELINE configs 4 and 5: Llama-3 8B / 70B shapes, random-init Q4_0
    "llama3-8b": dict(n_layer=32, hidden=4096, n_head=32, n_head_kv=8, head_dim=128, ffn=14336, vocab=128256,
                      ctx=4096),
    # the 8B shape with llama.cpp's Q4_K_M format mix (q4_k_m_types)
    "llama3-8b-q4_k_m": dict(n_layer=32, hidden=4096, n_head=32, n_head_kv=8, head_dim=128, ffn=14336,
                             vocab=128256, ctx=4096, mix="q4_k_m"),
    "llama3-70b": dict(n_layer=80, hidden=8192, n_head=64, n_head_kv=8, head_dim=128, ffn=28672, vocab=128256,
                       ctx=8192),
}
DECODE_STEPS, DECODE_WARMUP = 48, 4


def q4_k_m_types(P, n_layer):
    """Per-tensor formats of a llama.cpp Q4_K_M file: Q4_K, with attn_v and
    ffn_down in Q6_K in the first and last eighth of the layers and in every
    third layer between, and the output matrix in Q6_K."""
    t = [P.Q4_K] * P.dec_tensor_types(n_layer)
    t[P.TT_LM_HEAD] = P.Q6_K
    e = n_layer // 8
    for l in range(n_layer):
        if l < e or l >= n_layer - e or (l - e) % 3 == 2:
            t[P.tt_layer(l, P.TT_V)] = P.Q6_K
            t[P.tt_layer(l, P.TT_DOWN)] = P.Q6_K
    return t


def ktypes_section(torch, P, stream):
    """Batch-1 mat-vec of the K-quant formats (the team kernel) at the 8B
    decode shapes: GB/s of weight + activation bytes per launch, launches
    chained with PDL over weight copies rotating beyond 3x L2."""
    peak = peak_gbs()[0]
    out = {}
    shapes = (("gate_up", 4096, 28672), ("down", 14336, 4096), ("lm_head", 4096, 128256))
    for qt, qname in ((P.Q4_K, "q4_k"), (P.Q5_K, "q5_k"), (P.Q6_K, "q6_k")):
        out[qname] = {}
        for name, k, rows in shapes:
            nbytes_w = rows * (k // P.BLOCK_ELEMS[qt]) * P.BLOCK_BYTES[qt]
            copies = max(2, int(np.ceil(3 * L2_BYTES / nbytes_w)) + 1)
            ws = [torch.randint(0, 256, (nbytes_w,), dtype=torch.uint8, device="cuda") for _ in range(copies)]
            xq = P.q8_1_quantize(torch.from_numpy(W.activations(1, k, seed=k)).cuda())
            y = torch.empty(1, rows, device="cuda")
            reps = max(4, 32 // copies)
            g = capture(torch, lambda: [P.qmv(qt, ws[r % copies], rows, k, xq, 1, y=y, flags=P.QMV_PDL)
                                        for r in range(copies * reps)])
            time_graphs(torch, [g], 2, stream)
            n = 10
            us = time_graphs(torch, [g], n, stream) / (n * copies * reps) * 1e3
            nbytes = W.qmv_algorithmic_bytes(qt, rows, k, 1)
            out[qname][f"{name} {k}x{rows}"] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                                                "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
            del ws, g
    return out


def stats(values):
    """Median, min and max of a measurement repeated over rounds."""
    return {"median": round(statistics.median(values), 4), "min": round(min(values), 4),
            "max": round(max(values), 4), "rounds": len(values)}


DECODE_ROUNDS = 3
PARITY_STEPS = 8


def decode_parity(torch, P, m, cfg_kwargs, dec, stream, world, dist):
    """TP=N against TP=1 in the same run: every rank also builds the unsplit
    model (one GPU holds it beside its slice), both start from the same state
    and run PARITY_STEPS steps; each step the TP decoder is fed the TP=1
    token.  Reports whether every step picked the same token and the largest
    logit difference (each rank its vocabulary slice, max over ranks)
    relative to the TP=1 logits' largest magnitude."""
    ctx = m["ctx"]
    ref = P.Decoder(P.LlamaConfig(**cfg_kwargs), None)
    try:
        for d in (ref, dec):
            d.init_random(20261201)
            d.fill_kv(ctx, 7, 0.5)
            d.set_state(ctx, 1)
        off = dec.vocab_offset
        equal, worst = True, 0.0
        for _ in range(PARITY_STEPS):
            ref.step(1, stream)
            dec.step(1, stream)
            rpos, rtok = ref.state()
            pos, tok = dec.state()
            rl = ref.read(*ref.buffer(P.B_LOGITS)).view(np.float32)
            gl = dec.read(*dec.buffer(P.B_LOGITS)).view(np.float32)
            worst = max(worst, float(np.abs(gl - rl[off:off + gl.size]).max() / np.abs(rl).max()))
            equal = equal and tok == rtok and pos == rpos
            if tok != rtok:
                dec.set_state(pos, rtok)   # teacher-forced: the next step starts from the same token
    finally:
        ref.close()
    t = torch.tensor([worst, 0.0 if equal else 1.0], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {"steps": PARITY_STEPS, "tokens_equal": t[1].item() == 0.0, "max_logit_diff": round(t[0].item(), 8),
            "bound": 1e-2, "against": "the unsplit model on one GPU (every rank), same state, teacher-forced tokens"}


def decode_section(torch, P, stream, rank, world, dist, max_over_ranks, tp):
    """Configs 4/5: batch-1 decode tokens/s of the 8B and 70B shapes, the model
    row-split over the `world` ranks (TP=world; o and down all-reduced
    through NVLink peer memory, pushed from the mat-vec's epilogue).  KV
    prefilled to the config's context (N(0,1)*0.5 fp16); each step appends
    one row and attends over the whole cache, one CUDA graph per token
    replayed back to back; CUDA events, max over ranks, DECODE_ROUNDS rounds
    (median, min, max).  e2e additionally reads every token on the host.
    With world > 1 the 8B model also reports tp_parity (against the unsplit
    model) and the exchange's cost (the step minus the same slice shapes
    decoded alone on one GPU, per layer)."""
    out = {}
    peak, _ = peak_gbs()
    for name, m in DECODE_MODELS.items():
        ctx = m["ctx"]
        mix = q4_k_m_types(P, m["n_layer"]) if m.get("mix") == "q4_k_m" else None
        cfg_kwargs = dict(n_layer=m["n_layer"], hidden=m["hidden"], n_head=m["n_head"], n_head_kv=m["n_head_kv"],
                          head_dim=m["head_dim"], ffn=m["ffn"], vocab=m["vocab"],
                          max_ctx=ctx + DECODE_WARMUP + (DECODE_ROUNDS + 2) * DECODE_STEPS + PARITY_STEPS + 8,
                          wtype=P.Q4_K if mix else P.Q4_0, tensor_types=mix)
        dec = P.Decoder(P.LlamaConfig(**cfg_kwargs), tp)
        try:
            dec.init_random(20261201)
            dec.fill_kv(ctx, 7, 0.5)
            dec.set_state(ctx, 1)
            dec.step(DECODE_WARMUP, stream)
            torch.cuda.synchronize()
            per = []
            for _ in range(DECODE_ROUNDS):
                if dist is not None:
                    dist.barrier()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                dec.step(DECODE_STEPS, stream)
                b.record(stream)
                b.synchronize()
                per.append(max_over_ranks(a.elapsed_time(b)) / DECODE_STEPS)
            ms = statistics.median(per)
            t0 = time.perf_counter()
            for _ in range(DECODE_STEPS):
                dec.step(1, stream)
                dec.state()               # synchronises and reads the token on the host
            e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3) / DECODE_STEPS
            pos, tok = dec.state()
            kv_rank = m["n_layer"] * 2 * (m["n_head_kv"] // world) * m["head_dim"] * 2 * (ctx + DECODE_WARMUP
                                                                                        + DECODE_STEPS)
            rank_bytes = dec.weight_bytes_per_token + kv_rank
            row = {"tok_s": round(1e3 / ms, 2), "ms_per_token": round(ms, 4),
                   "tok_s_rounds": stats([1e3 / v for v in per]), "context": ctx, "tp": world,
                   "bytes_per_token_per_gpu": rank_bytes,
                   "hbm_frac_per_gpu": round(rank_bytes / (ms / 1e3) / 1e9 / peak, 4),
                   "e2e_tok_s": round(1e3 / e2e_ms, 2), "last_token": tok, "position": pos,
                   "exchange": ("peer memory, pushed from the o/down mat-vec epilogue" if world > 1 else "none")}
            if world > 1 and name == "llama3-8b":
                row["tp_parity"] = decode_parity(torch, P, m, cfg_kwargs, dec, stream, world, dist)
                row["exchange_us_per_layer"] = exchange_cost(torch, P, m, ms, stream, world, max_over_ranks)
            out[name] = row
        finally:
            dec.close()   # releases the graph (and any NCCL calls in it) before the communicator
        P.check(P.device_error())
    return out


def exchange_cost(torch, P, m, ms_tp, stream, world, max_over_ranks):
    """Per layer: the TP=world step minus the same slice shapes (n_head/N,
    n_head_kv/N, ffn/N, vocab/N) decoded alone on this GPU with no exchange."""
    cfg = P.LlamaConfig(m["n_layer"], m["hidden"], m["n_head"] // world, m["n_head_kv"] // world, m["head_dim"],
                        m["ffn"] // world, m["vocab"] // world, m["ctx"] + DECODE_WARMUP + DECODE_STEPS + 8)
    dec = P.Decoder(cfg, None)
    try:
        dec.init_random(3)
        dec.fill_kv(m["ctx"], 7, 0.5)
        dec.set_state(m["ctx"], 1)
        dec.step(DECODE_WARMUP, stream)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dec.step(DECODE_STEPS, stream)
        b.record(stream)
        b.synchronize()
        ms_slice = max_over_ranks(a.elapsed_time(b)) / DECODE_STEPS
    finally:
        dec.close()
    return {"slice_alone_ms": round(ms_slice, 4), "tp_ms": round(ms_tp, 4),
            "us_per_layer": round((ms_tp - ms_slice) * 1e3 / m["n_layer"], 3)}


def collective_section(torch, P, tp, stream, world, dist):
    """All-reduce latency at the per-layer exchange sizes (fp32 sum of 16, 32
    and 64 KB), 64 calls captured in a graph: the library's
    p100_tp_allreduce_sum as the headline uses it (one kernel over NVLink peer
    memory where tp.peer) and ncclAllReduce (a second communicator joined with
    P100_TP_ALLREDUCE=nccl, closed here).  Bus bandwidth 2 (N-1)/N x bytes /
    time, the analogue of the reference's p2p_bandwidth benchmark for this
    layout's only collective."""
    box = [P.tp_unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(box, src=0)
    saved = os.environ.get("P100_TP_ALLREDUCE")
    os.environ["P100_TP_ALLREDUCE"] = "nccl"
    try:
        nccl_tp = P.TP(box[0], world, tp.rank, torch.cuda.current_device())
    finally:
        if saved is None:
            del os.environ["P100_TP_ALLREDUCE"]
        else:
            os.environ["P100_TP_ALLREDUCE"] = saved
    out = {"p100_tp_path": "peer memory" if tp.peer else "nccl"}
    try:
        for label, h in (("p100_tp_allreduce", tp), ("nccl_allreduce", nccl_tp)):
            per_size = {}
            for nbytes in (16384, 32768, 65536):
                buf = torch.ones(nbytes // 4, device="cuda")
                # the current stream: inside capture that is the capturing stream
                g = capture(torch, lambda h=h, buf=buf: [h.allreduce_sum(buf) for _ in range(64)])
                time_graphs(torch, [g], 3, stream)
                per = [time_graphs(torch, [g], 5, stream) / (5 * 64) * 1e3 for _ in range(3)]
                us = statistics.median(per)
                per_size[f"{nbytes // 1024}KB"] = {
                    "us": round(us, 3), "busbw_GBs": round(2 * (world - 1) / world * nbytes / us / 1e3, 3),
                    "us_rounds": stats(per)}
                del g   # before the communicator closes
            out[label] = per_size
        torch.cuda.synchronize()
    finally:
        nccl_tp.close()
    return out


def c2_grid(torch, P, stream):
    """Config 2: every layer shape x Q4_0/Q8_0/Q4_K x batch 1, 2, 4, 8, 16,
    one C-ABI call per launch, graph-replayed back to back with PDL over
    rotating weight copies that together exceed 3x L2.  Batch 1 runs the team
    kernel, batch 2-16 the tensor-core kernel (one launch for all columns).
    GB/s counts the algorithmic bytes (weights + activations + outputs)."""
    peak = peak_gbs()[0]
    out = {}
    for qtype, tname in ((W.Q4_0, "Q4_0"), (W.Q8_0, "Q8_0"), (W.Q4_K, "Q4_K")):
        per_type = {}
        for si, (name, k, rows) in enumerate(SHAPES):
            base = torch.from_numpy(W.weights(qtype, rows, k, seed=5000 + 31 * si + qtype)).cuda()
            copies = max(4, int(np.ceil(3 * L2_BYTES / base.numel())) + 1)
            ws = [base] + [base.clone() for _ in range(copies - 1)]
            n_in_graph = max(16, copies)
            per_shape = {}
            for b in (1, 2, 4, 8, 16):
                xqb = P.q8_1_quantize(torch.from_numpy(W.activations(b, k, seed=4000 + b + k)).cuda())
                yb = torch.empty(b, rows, dtype=torch.float32, device="cuda")
                g = capture(torch, lambda xqb=xqb, yb=yb, b=b: [
                    P.qmv(qtype, ws[r % copies], rows, k, xqb, b, y=yb, flags=P.QMV_PDL) for r in range(n_in_graph)])
                time_graphs(torch, [g], 2, stream)
                reps = 5
                us = time_graphs(torch, [g], reps, stream) / (reps * n_in_graph) * 1e3
                nbytes = W.qmv_algorithmic_bytes(qtype, rows, k, b)
                per_shape[str(b)] = {"us": round(us, 3), "GB/s": round(nbytes / (us / 1e6) / 1e9, 1),
                                     "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4)}
                del g
            per_type[f"{name} {k}x{rows}"] = per_shape
            del ws, base
        out[tname] = per_type
    torch.cuda.synchronize()
    P.check(P.device_error())
    return out


def kernel_only(args):
    """Eager launches of one kernel over rotating inputs larger than L2 — the
    small cases for ncu captures: the target mat-vec at batch 1 or 16 (5 weight
    copies, 165 MB) or FA decode at 32K context (2 K/V copies, 268 MB) or 4K."""
    import torch
    import p100_b200 as P
    if args.kernel_only == "decode":
        # the 8B decoder (config 4): warmup + steps tokens, 324 launches each
        m = DECODE_MODELS["llama3-8b"]
        cfg = P.LlamaConfig(m["n_layer"], m["hidden"], m["n_head"], m["n_head_kv"], m["head_dim"], m["ffn"], m["vocab"],
                            m["ctx"] + args.warmup + args.steps + 8)
        dec = P.Decoder(cfg)
        dec.init_random(20261201)
        dec.fill_kv(m["ctx"], 7, 0.5)
        dec.set_state(m["ctx"], 1)
        dec.step(args.warmup + args.steps, torch.cuda.current_stream())
        pos, tok = dec.state()
        dec.close()
        P.check(P.device_error())
        print(json.dumps({"kernel_only": "decode llama3-8b ctx 4096", "steps": args.warmup + args.steps,
                          "position": pos, "token": tok}))
        return 0
    if args.kernel_only in ("fa", "fa4096", "faq8", "faq4"):
        seq = 4096 if args.kernel_only == "fa4096" else 32768
        kv_type = {"faq8": P.KV_Q8_0, "faq4": P.KV_Q4_0}.get(args.kernel_only, P.KV_F16)
        q, k, v = W.attention_inputs(1, 32, 8, seq, 128, seed=seq)
        if kv_type != P.KV_F16:
            k = W.kv_cache_blocks(kv_type, 1, 8, seq, 128, seed=seq + 1)
            v = W.kv_cache_blocks(kv_type, 1, 8, seq, 128, seed=seq + 2)
        qd = torch.from_numpy(q).cuda()
        kd = [torch.from_numpy(k).cuda() for _ in range(2)]
        vd = [torch.from_numpy(v).cuda() for _ in range(2)]
        desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=seq, kv_type=kv_type)
        ws = P.fa_workspace(desc)
        for i in range(args.warmup + args.steps):
            P.fa_decode(desc, qd, kd[i % 2], vd[i % 2], ws=ws)
        torch.cuda.synchronize()
        P.check(P.device_error())
        print(json.dumps({"kernel_only": f"fa_decode 32/8 heads d128 ctx {seq} kv_type {kv_type}",
                          "launches": args.warmup + args.steps}))
        return 0
    _, k, rows = TARGET
    batch = 16 if args.kernel_only == "qmvb" else 1
    if args.kernel_only == "h16":
        # the h16 path (HFMA2 chain 16) on the target shape, 5 copies (165 MB > L2)
        ws = [torch.from_numpy(W.weights(W.Q4_0, rows, k, seed=s_)).cuda() for s_ in range(5)]
        h, ss = P.h16_prepare(torch.from_numpy(W.activations(1, k, seed=2)).cuda())
        y = torch.empty(1, rows, device="cuda")
        for i in range(args.warmup + args.steps):
            P.qmv_h16(W.Q4_0, ws[i % 5], rows, k, h, ss, 1, 16, y=y)
        torch.cuda.synchronize()
        P.check(P.device_error())
        print(json.dumps({"kernel_only": f"qmv_h16 Q4_0 {k}x{rows} chain 16", "launches": args.warmup + args.steps}))
        return 0
    if args.kernel_only == "qmvtc":
        # the tcgen05 batched kernel: Q4_K on the target shape at batch 8, 5 copies (165 MB > L2)
        ws = [torch.from_numpy(W.weights(W.Q4_K, rows, k, seed=s_)).cuda() for s_ in range(5)]
        xq = P.q8_1_quantize(torch.from_numpy(W.activations(8, k, seed=2)).cuda())
        y = torch.empty(8, rows, device="cuda")
        for i in range(args.warmup + args.steps):
            P.qmv(W.Q4_K, ws[i % 5], rows, k, xq, 8, y=y, flags=P.QMV_TC)
        torch.cuda.synchronize()
        P.check(P.device_error())
        print(json.dumps({"kernel_only": f"qmv_tc Q4_K {k}x{rows} batch 8", "launches": args.warmup + args.steps}))
        return 0
    if args.kernel_only == "qmv6k":
        # the Q6_K LM head of a Q4_K_M 8B model: 4096 x 128256, 431 MB > L2
        k, rows = 4096, 128256
        ws = [torch.from_numpy(W.weights(W.Q6_K, rows, k, seed=s_)).cuda() for s_ in (1, 2)]
        xq = P.q8_1_quantize(torch.from_numpy(W.activations(1, k, seed=2)).cuda())
        y = torch.empty(1, rows, device="cuda")
        for i in range(args.warmup + args.steps):
            P.qmv(W.Q6_K, ws[i % 2], rows, k, xq, 1, y=y)
        torch.cuda.synchronize()
        P.check(P.device_error())
        print(json.dumps({"kernel_only": f"qmv Q6_K {k}x{rows} batch 1", "launches": args.warmup + args.steps}))
        return 0
    base = torch.from_numpy(W.weights(W.Q4_0, rows, k, seed=1)).cuda()
    ws = [base] + [base.clone() for _ in range(4)]
    xq = P.q8_1_quantize(torch.from_numpy(W.activations(batch, k, seed=2)).cuda())
    y = torch.empty(batch, rows, device="cuda")
    for i in range(args.warmup + args.steps):
        P.qmv(W.Q4_0, ws[i % len(ws)], rows, k, xq, batch, y=y)
    torch.cuda.synchronize()
    P.check(P.device_error())
    print(json.dumps({"kernel_only": f"qmv Q4_0 {k}x{rows} batch {batch}", "launches": args.warmup + args.steps}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the 8B/70B decode section")
    ap.add_argument("--kernel-only",
                    choices=["qmv", "qmvb", "qmvtc", "qmv6k", "h16", "fa", "fa4096", "faq8", "faq4", "decode"],
                    help="one kernel's launches only (ncu cases); qmvb = the target shape at batch 16, "
                         "qmvtc = the target shape in Q4_K at batch 8 on the tcgen05 kernel, "
                         "h16 = the target shape on the h16 path, "
                         "qmv6k = a Q6_K 4096x128256 LM head at batch 1, "
                         "fa = 32768 keys, fa4096 = 4096 keys, faq8 / faq4 = 32768 keys of q8_0 / q4_0 K/V")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.kernel_only:
        return kernel_only(args)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

    import torch
    import p100_b200 as P

    torch.cuda.set_device(local)
    dist = None
    tp = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    P.check(P.device_check(local))
    stream = torch.cuda.current_stream()
    if world > 1:
        box = [P.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = P.TP(box[0], world, rank, local)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # The full layer step (every rank the whole shapes; at N > 1 the
    # replicated weak-scaling figure): one host-generated set per shape,
    # replicated on the device into `copies` copies so successive steps
    # rotate through more than 3x L2.
    per_copy = sum(W.weights(W.Q4_0, 1, k, 0).size * rows for _, k, rows in SHAPES)
    copies = max(4, int(np.ceil(3 * L2_BYTES / per_copy)) + 1)
    wdev = []
    for si, (name, k, rows) in enumerate(SHAPES):
        base = torch.from_numpy(W.weights(W.Q4_0, rows, k, seed=1000 + si + 17 * rank)).cuda()
        wdev.append([base] + [base.clone() for _ in range(copies - 1)])
    xs = [torch.from_numpy(W.activations(1, k, seed=2000 + si)).cuda() for si, (_, k, _) in enumerate(SHAPES)]
    xqs = [torch.empty(P.q8_1_bytes(k, 1), dtype=torch.uint8, device="cuda") for _, k, _ in SHAPES]
    ys = [torch.empty(1, rows, dtype=torch.float32, device="cuda") for _, _, rows in SHAPES]
    launches_per_step = 2 * len(SHAPES)

    def step_body(c):
        # p100_qmv_f32 per shape: the Q8_1 quantiser, a programmatic dependent
        # of the previous mat-vec (launched during its tail, reading x after
        # it ends), then the mat-vec as the quantiser's programmatic dependent
        # (its weights stream in while the quantiser runs).  Measured 26.7 us
        # a step against 30.7 with the quantiser launched plainly and 38.9
        # with the quantisation fused into every mat-vec CTA.
        for si, (name, k, rows) in enumerate(SHAPES):
            P.qmv_f32(W.Q4_0, wdev[si][c], rows, k, xs[si], x_q8_1=xqs[si], y=ys[si], flags=P.QMV_PDL)

    graphs = [capture(torch, lambda c=c: step_body(c)) for c in range(copies)]

    # N > 1: the same global layer step split over the ranks (the headline,
    # strong scaling): q/o and down split along k (their outputs are partial
    # sums, all-reduced in the timed region), k/v and gate/up by rows.
    split_graphs, split_copies, split_launches = None, 0, 0
    if world > 1:
        plan = []
        for si, (name, k, rows) in enumerate(SHAPES):
            ksplit = name in ("q/o", "down")
            plan.append((ksplit, k // world if ksplit else k, rows if ksplit else rows // world))
        split_per_copy = sum(W.weights(W.Q4_0, 1, lk, 0).size * lr for _, lk, lr in plan)
        split_copies = max(4, int(np.ceil(3 * L2_BYTES / split_per_copy)) + 1)
        sw, sx, sq, sy = [], [], [], []
        for si, (ksplit, lk, lr) in enumerate(plan):
            base = torch.from_numpy(W.weights(W.Q4_0, lr, lk, seed=5000 + si + 17 * rank)).cuda()
            sw.append([base] + [base.clone() for _ in range(split_copies - 1)])
            sx.append(torch.from_numpy(W.activations(1, lk, seed=6000 + si + 17 * rank)).cuda())
            sq.append(torch.empty(P.q8_1_bytes(lk, 1), dtype=torch.uint8, device="cuda"))
            sy.append(torch.empty(1, lr, dtype=torch.float32, device="cuda"))

        def split_body(c):
            for si, (ksplit, lk, lr) in enumerate(plan):
                P.qmv_f32(W.Q4_0, sw[si][c], lr, lk, sx[si], x_q8_1=sq[si], y=sy[si], flags=P.QMV_PDL)
                if ksplit:
                    tp.allreduce_sum(sy[si])   # the current (capturing) stream

        split_graphs = [capture(torch, lambda c=c: split_body(c)) for c in range(split_copies)]
        split_launches = 2 * len(SHAPES)

    # The target shape alone (the roofline): a graph of 4*copies back-to-back
    # launches over the rotating copies, chained with PDL and isolated.
    ti = [i for i, sh in enumerate(SHAPES) if sh == TARGET][0]
    P.q8_1_quantize(xs[ti], out=xqs[ti])
    n_in_graph = 4 * copies
    target_graphs = {}
    for mode, flags in (("chained", P.QMV_PDL), ("isolated", 0)):
        target_graphs[mode] = capture(torch, lambda flags=flags: [
            P.qmv(W.Q4_0, wdev[ti][r % copies], TARGET[2], TARGET[1], xqs[ti], 1, y=ys[ti], flags=flags)
            for r in range(n_in_graph)])
    head_graphs = split_graphs if split_graphs else graphs
    time_graphs(torch, graphs, args.warmup, stream)
    if split_graphs:
        time_graphs(torch, split_graphs, args.warmup, stream)
    for g in target_graphs.values():
        time_graphs(torch, [g], 3, stream)
    barrier()
    torch.cuda.synchronize()

    # Interleaved rounds: each round times exactly --steps steps of the
    # headline (barrier and synchronisation on both sides, max over ranks),
    # then the replicated step (N > 1) and the target shape chained and
    # isolated; rounds repeat until the window covers a second (at least 3).
    head_ms, rep_ms, chained_us, isolated_us = [], [], [], []
    reps = 10
    t_start = time.perf_counter()
    with ClockSampler(local) as clocks:
        while True:
            barrier()
            torch.cuda.synchronize()
            head_ms.append(max_over_ranks(time_graphs(torch, head_graphs, args.steps, stream)))
            barrier()
            if split_graphs:
                rep_ms.append(max_over_ranks(time_graphs(torch, graphs, args.steps, stream)))
            chained_us.append(time_graphs(torch, [target_graphs["chained"]], reps, stream) / (reps * n_in_graph) * 1e3)
            isolated_us.append(time_graphs(torch, [target_graphs["isolated"]], reps, stream) / (reps * n_in_graph) * 1e3)
            window = max_over_ranks(time.perf_counter() - t_start)
            if len(head_ms) >= 3 and (window >= 1.0 or len(head_ms) >= 200):
                break
    window_s = time.perf_counter() - t_start
    del target_graphs
    per_step = step_bytes()
    ms = statistics.median(head_ms)
    value = per_step * args.steps / (ms / 1e3) / 1e9 if split_graphs else per_step * world * args.steps / (ms / 1e3) / 1e9
    head_gbs = [per_step * (1 if split_graphs else world) * args.steps / (v / 1e3) / 1e9 for v in head_ms]
    replicated = None
    if split_graphs:
        rgbs = [per_step * world * args.steps / (v / 1e3) / 1e9 for v in rep_ms]
        replicated = {"value": round(statistics.median(rgbs), 2), "unit": "GB/s", "scaling": "weak",
                      "rounds": stats(rgbs),
                      "form": "every rank streams the full layer shapes (its own weights), no data-path collective"}
    target_us, target_us_isolated = statistics.median(chained_us), statistics.median(isolated_us)

    # Each shape alone (chained and isolated), for the record.
    shape_gbs = {}
    for si, (name, k, rows) in enumerate(SHAPES):
        P.q8_1_quantize(xs[si], out=xqs[si])
        per = {}
        for mode, flags in (("chained", P.QMV_PDL), ("isolated", 0)):
            g = capture(torch, lambda si=si, k=k, rows=rows, flags=flags: [
                P.qmv(W.Q4_0, wdev[si][r % copies], rows, k, xqs[si], 1, y=ys[si], flags=flags)
                for r in range(n_in_graph)])
            time_graphs(torch, [g], 3, stream)
            per[mode] = time_graphs(torch, [g], 20, stream) / (20 * n_in_graph) * 1e3
            del g
        nbytes = W.qmv_algorithmic_bytes(W.Q4_0, rows, k, 1)
        shape_gbs[f"{name} {k}x{rows}"] = {
            "us": round(per["chained"], 3), "GB/s": round(nbytes / (per["chained"] / 1e6) / 1e9, 1),
            "us_isolated": round(per["isolated"], 3),
            "GB/s_isolated": round(nbytes / (per["isolated"] / 1e6) / 1e9, 1)}

    batch_sweep = c2_grid(torch, P, stream) if rank == 0 else None

    # End to end through the C-ABI with host buffers, on the headline's step
    # (the split step at N > 1): each step copies its activations in from
    # pinned memory, runs (with its all-reduces), copies y out and
    # synchronises before the host reads the result.  "graph": the calls
    # captured once and replayed (a decode loop's form); "eager": the calls
    # issued every step.  Three rounds, the median.
    if split_graphs:
        e_plan = [(sw[si], lk, lr, ksplit) for si, (ksplit, lk, lr) in enumerate(plan)]
        e_copies = split_copies
    else:
        e_plan = [(wdev[si], k, rows, False) for si, (_, k, rows) in enumerate(SHAPES)]
        e_copies = copies
    xh = [torch.from_numpy(W.activations(1, lk, seed=3000 + si)).pin_memory() for si, (_, lk, _, _) in enumerate(e_plan)]
    yh = [torch.empty(1, lr, dtype=torch.float32).pin_memory() for _, _, lr, _ in e_plan]
    xd = [torch.empty(1, lk, dtype=torch.float32, device="cuda") for _, lk, _, _ in e_plan]
    eq = [torch.empty(P.q8_1_bytes(lk, 1), dtype=torch.uint8, device="cuda") for _, lk, _, _ in e_plan]
    ey = [torch.empty(1, lr, dtype=torch.float32, device="cuda") for _, _, lr, _ in e_plan]
    h2d = sum(t.numel() * 4 for t in xh)
    d2h = sum(t.numel() * 4 for t in yh)

    def e2e_body(c):
        for si, (wl, lk, lr, ksplit) in enumerate(e_plan):
            xd[si].copy_(xh[si], non_blocking=True)
            P.qmv_f32(W.Q4_0, wl[c], lr, lk, xd[si], x_q8_1=eq[si], y=ey[si], flags=P.QMV_PDL)
            if ksplit:
                tp.allreduce_sum(ey[si])   # the current (capturing) stream
            yh[si].copy_(ey[si], non_blocking=True)

    e2e_graphs = [capture(torch, lambda c=c: e2e_body(c)) for c in range(e_copies)]
    checksum = 0.0

    def e2e_run(n, eager):
        nonlocal checksum
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for i in range(n):
            if eager:
                e2e_body(i % e_copies)
            else:
                e2e_graphs[i % e_copies].replay()
            stream.synchronize()
            checksum += float(yh[0][0, 0])      # the host reads the step's result
        e.record(stream)
        torch.cuda.synchronize()
        return s.elapsed_time(e)

    e2e_run(args.warmup, False)
    e2e_run(args.warmup, True)
    e2e_rounds, e2e_eager_rounds = [], []
    for _ in range(3):
        barrier()
        e2e_rounds.append(max_over_ranks(e2e_run(args.steps, False)))
        barrier()
        e2e_eager_rounds.append(max_over_ranks(e2e_run(args.steps, True)))
    job_bytes = per_step * (1 if split_graphs else world) * args.steps
    e2e_value = job_bytes / (statistics.median(e2e_rounds) / 1e3) / 1e9
    e2e_eager = job_bytes / (statistics.median(e2e_eager_rounds) / 1e3) / 1e9
    del e2e_graphs
    fa = fa_section(torch, P, stream) if rank == 0 else None
    h16 = h16_section(torch, P, stream) if rank == 0 else None
    kvq = kv_quant_section(torch, P, stream) if rank == 0 else None
    kq = ktypes_section(torch, P, stream) if rank == 0 else None
    P.check(P.device_error())
    decode = decode_section(torch, P, stream, rank, world, dist, max_over_ranks, tp) if not args.no_decode else None
    collective = collective_section(torch, P, tp, stream, world, dist) if tp is not None else None

    peak, peak_kind = peak_gbs()
    target_bytes = W.qmv_algorithmic_bytes(W.Q4_0, TARGET[2], TARGET[1], 1)
    achieved = target_bytes / (target_us / 1e6) / 1e9
    split_desc = ("TP=%d: q/o and down split along k (partial sums, each all-reduced with p100_tp_allreduce_sum "
                  "(%s) in the timed region), k/v and gate/up split by rows"
                  % (world, "one kernel over NVLink peer memory" if tp is not None and tp.peer else "ncclAllReduce"))
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong" if split_graphs else "weak",
        "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
        "rounds": dict(stats(head_gbs), window_s=round(window_s, 3), steps_per_round=args.steps),
        "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": 1,
                   "parallelism": split_desc if split_graphs else "1 GPU",
                   "l2": f"inputs larger than L2: {split_copies if split_graphs else copies} rotating weight copies",
                   "launch": "one p100_qmv_f32 call per shape (Q8_1 quantiser + mat-vec, PDL-chained), captured into one CUDA graph per weight copy, replayed per step"},
        "roofline": {"bound": "hbm", "kernel": "qmv_team_kernel<Q4_0> gate/up 4096x14336",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": ncu_traffic("qmv_q4_0_4096x14336"), "algorithmic_bytes": target_bytes,
                     "us_per_launch": round(target_us, 3),
                     "us_rounds": stats(chained_us),
                     "frac_rounds": stats([target_bytes / (u / 1e6) / 1e9 / peak for u in chained_us]),
                     "timing": "CUDA events over graph replays of back-to-back launches chained with PDL, "
                               "interleaved with the headline's rounds",
                     "isolated_us_per_launch": round(target_us_isolated, 3),
                     "isolated_frac": round(target_bytes / (target_us_isolated / 1e6) / 1e9 / peak, 4)},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "form": "graph replay + stream sync + host read per step (median of 3 rounds)",
                "eager_value": round(e2e_eager, 2)},
        "gpu_launches": (split_launches if split_graphs else launches_per_step) * args.steps * len(head_ms),
        "gpu_launches_note": "the library's mat-vec and quantiser kernels in the headline's timed rounds (all-reduce "
                             "kernels not counted)",
        "replicated": replicated,
        "shapes": shape_gbs,
        "batch_sweep": batch_sweep,
        "fa_decode": fa,
        "h16_qmv": h16,
        "quantised_kv": kvq,
        "ktypes_qmv": kq,
        "decode": decode,
        "collective": collective,
        "clocks": clocks.summary(),
        "checksum": round(checksum, 3),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_sample()
    if rank == 0:
        print(json.dumps(result), flush=True)
    # every graph that holds NCCL calls goes before the communicator (its
    # destroy waits for them): head_graphs aliases split_graphs
    del graphs, split_graphs, head_graphs
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if tp is not None:
        tp.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
