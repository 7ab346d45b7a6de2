"""Seeded synthetic inputs in the distributions of the benchmark configurations.

Host-side numpy generators (one seed per tensor) for the mat-vec and attention
workloads: there is no dataset or checkpoint behind this path, so these stand
in for model weights, activations and a prefilled KV cache.

* Q4_0: per block d = fp16(|N(0,1)| * 0.02), 32 codes uniform in 0..15
  (value d * (code - 8)); low nibble of byte i is element i, high nibble is
  element i + 16 (include/p100/qmv.h:6, qmv_model.cpp:82).
* Q8_0: d as above, codes uniform in -127..127.
* Q4_K: d, dmin = fp16(|N(0,1)| * 0.02), 12 packed scale bytes uniform in
  0..255 (so every 6-bit scale/min is uniform), 128 nibble bytes uniform.
* Q5_K: as Q4_K, plus the 32 high-bit bytes uniform.
* Q6_K: the 128 low-nibble, 64 high-bit and 16 int8 scale bytes uniform,
  d = fp16(|N(0,1)| * 0.02).
* activations ~ N(0,1) fp32; K/V cache fp16 N(0,1) * 0.5; q ~ N(0,1).
"""
from __future__ import annotations

import numpy as np

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 4
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}

# Llama-3-8B layer shapes of the mat-vec sweep, (name, k, rows).
LLAMA3_8B_SHAPES = [("q/o", 4096, 4096), ("k/v", 4096, 1024), ("gate/up", 4096, 14336), ("down", 14336, 4096)]


def _scales(rng, shape):
    return (np.abs(rng.standard_normal(shape)) * 0.02).astype(np.float16)


def weights(qtype, rows, k, seed):
    """rows x k weight matrix of qtype as GGUF block bytes (uint8, row-major)."""
    rng = np.random.default_rng(seed)
    be = BLOCK_ELEMS[qtype]
    if k % be:
        raise ValueError("whole weight blocks required")
    nb = k // be
    if qtype == Q4_0:
        out = np.empty((rows, nb, 18), np.uint8)
        out[..., :2] = _scales(rng, (rows, nb)).view(np.uint8).reshape(rows, nb, 2)
        codes = rng.integers(0, 16, (rows, nb, 32), dtype=np.uint8)
        out[..., 2:] = codes[..., :16] | (codes[..., 16:] << 4)
    elif qtype == Q8_0:
        out = np.empty((rows, nb, 34), np.uint8)
        out[..., :2] = _scales(rng, (rows, nb)).view(np.uint8).reshape(rows, nb, 2)
        out[..., 2:] = rng.integers(-127, 128, (rows, nb, 32), dtype=np.int8).view(np.uint8)
    elif qtype in (Q4_K, Q5_K):
        bb = BLOCK_BYTES[qtype]
        out = np.empty((rows, nb, bb), np.uint8)
        out[..., 0:2] = _scales(rng, (rows, nb)).view(np.uint8).reshape(rows, nb, 2)
        out[..., 2:4] = _scales(rng, (rows, nb)).view(np.uint8).reshape(rows, nb, 2)
        out[..., 4:] = rng.integers(0, 256, (rows, nb, bb - 4), dtype=np.uint8)
    else:   # Q6_K: ql, qh, int8 scales uniform; d last
        out = np.empty((rows, nb, 210), np.uint8)
        out[..., :208] = rng.integers(0, 256, (rows, nb, 208), dtype=np.uint8)
        out[..., 208:] = _scales(rng, (rows, nb)).view(np.uint8).reshape(rows, nb, 2)
    return out.reshape(-1)


def activations(batch, k, seed):
    return np.random.default_rng(seed).standard_normal((batch, k)).astype(np.float32)


def attention_inputs(batch, n_head_q, n_head_kv, seq_kv, d, seed):
    """q fp32 [B,Hq,1,D]; K, V fp16 [B,Hkv,S,D] ~ N(0,1)*0.5."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((batch, n_head_q, 1, d)).astype(np.float32)
    k = (rng.standard_normal((batch, n_head_kv, seq_kv, d), dtype=np.float32) * 0.5).astype(np.float16)
    v = (rng.standard_normal((batch, n_head_kv, seq_kv, d), dtype=np.float32) * 0.5).astype(np.float16)
    return q, k, v


def qmv_algorithmic_bytes(qtype, rows, k, batch):
    """Weight bytes + fp32 activations + fp32 outputs (bin/mm-gbps.py:51-57)."""
    return rows * (k // BLOCK_ELEMS[qtype]) * BLOCK_BYTES[qtype] + batch * k * 4 + batch * rows * 4


def fa_algorithmic_bytes(batch, n_head_q, n_head_kv, seq_kv, d, kv_type=0):
    """K and V read once (fp16, or q8_0 / q4_0 blocks: 34 / 18 bytes per 32
    values) + fp32 q and O (+ LSE)."""
    kv_row = d * 2 if kv_type == 0 else d // 32 * (34 if kv_type == 1 else 18)
    return batch * n_head_kv * seq_kv * kv_row * 2 + batch * n_head_q * d * 4 * 2 + batch * n_head_q * 4


def kv_cache_blocks(kv_type, batch, n_head_kv, seq_kv, d, seed):
    """A q8_0 / q4_0 K/V cache [B,Hkv,S,D/32*bb] of N(0,1)*0.5 rows for
    benchmarks, quantised on the host by ggml's block rule (x / (max|x| / 127)
    rounded for q8_0; trunc(x / (v / -8) + 8.5) clamped to 15, v the value of
    largest |x|, for q4_0), vectorised with numpy; the parity tests use the
    oracle's exact quantiser instead."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((batch * n_head_kv * seq_kv * d // 32, 32), dtype=np.float32) * 0.5)
    if kv_type == 1:
        dsc = np.abs(x).max(axis=1) / np.float32(127)
        idv = np.where(dsc != 0, np.float32(1) / np.where(dsc != 0, dsc, 1), 0).astype(np.float32)
        t = x * idv[:, None]
        q = np.trunc(t + np.copysign(np.float32(0.5), t)).astype(np.int8).view(np.uint8)
    else:
        j = np.abs(x).argmax(axis=1)
        vmax = x[np.arange(x.shape[0]), j]
        dsc = vmax / np.float32(-8)
        idv = np.where(dsc != 0, np.float32(1) / np.where(dsc != 0, dsc, 1), 0).astype(np.float32)
        c = np.minimum(15, np.trunc(x * idv[:, None] + np.float32(8.5))).astype(np.uint8)
        q = c[:, :16] | (c[:, 16:] << 4)
    blocks = np.concatenate([dsc.astype(np.float16).view(np.uint8).reshape(-1, 2), q], axis=1)
    return blocks.reshape(batch, n_head_kv, seq_kv, -1)
