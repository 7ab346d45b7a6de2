"""ggml's Q5_K and Q6_K super-blocks in the oracle (CPU).

The reference's contract has Q4_0 / Q8_0 / Q4_K only, so these two formats
have no golden vectors there.  The oracle's slab decoding
(oracle/p100_oracle.cpp slab_of) is checked instead against an independent
numpy restatement written in the loop structure of ggml's published
dequantize_row_q5_K / dequantize_row_q6_K (64- and 128-value groups, not
32-value slabs), and its q81 dot against the exact FP64 dot within the
reference's normalised tolerance."""
import numpy as np
import pytest

from conftest import QMV_NORM_TOL

import oracle
from p100_b200 import workloads as W


def scale_min_k4(scales, j):
    """get_scale_min_k4 for super-blocks [n, 12] -> (sc, mn) [n]."""
    s = scales.astype(np.int64)
    if j < 4:
        return s[:, j] & 63, s[:, j + 4] & 63
    return (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4), (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)


def numpy_dequant(qtype, raw):
    blk = raw.reshape(-1, W.BLOCK_BYTES[qtype])
    n = blk.shape[0]
    y = np.zeros((n, 256), np.float64)
    if qtype == W.Q5_K:
        d = blk[:, 0:2].copy().view(np.float16).astype(np.float64)[:, 0]
        dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float64)[:, 0]
        scales, qh, qs = blk[:, 4:16], blk[:, 16:48].astype(np.int64), blk[:, 48:176].astype(np.int64)
        for j in range(4):                      # 64 values per group
            sc1, m1 = scale_min_k4(scales, 2 * j)
            sc2, m2 = scale_min_k4(scales, 2 * j + 1)
            ql = qs[:, 32 * j:32 * j + 32]
            u1, u2 = 1 << (2 * j), 2 << (2 * j)
            y[:, 64 * j:64 * j + 32] = (d * sc1)[:, None] * ((ql & 15) + np.where(qh & u1, 16, 0)) - (dmin * m1)[:, None]
            y[:, 64 * j + 32:64 * j + 64] = (d * sc2)[:, None] * ((ql >> 4) + np.where(qh & u2, 16, 0)) - (dmin * m2)[:, None]
    else:
        d = blk[:, 208:210].copy().view(np.float16).astype(np.float64)[:, 0]
        for n128 in range(2):                   # 128 values per group
            ql = blk[:, 64 * n128:64 * n128 + 64].astype(np.int64)
            qh = blk[:, 128 + 32 * n128:128 + 32 * n128 + 32].astype(np.int64)
            sc = blk[:, 192 + 8 * n128:200 + 8 * n128].view(np.int8).astype(np.int64)
            for l in range(32):
                is_ = l // 16
                q1 = ((ql[:, l] & 15) | (((qh[:, l] >> 0) & 3) << 4)) - 32
                q2 = ((ql[:, l + 32] & 15) | (((qh[:, l] >> 2) & 3) << 4)) - 32
                q3 = ((ql[:, l] >> 4) | (((qh[:, l] >> 4) & 3) << 4)) - 32
                q4 = ((ql[:, l + 32] >> 4) | (((qh[:, l] >> 6) & 3) << 4)) - 32
                base = 128 * n128
                y[:, base + l] = d * sc[:, is_ + 0] * q1
                y[:, base + l + 32] = d * sc[:, is_ + 2] * q2
                y[:, base + l + 64] = d * sc[:, is_ + 4] * q3
                y[:, base + l + 96] = d * sc[:, is_ + 6] * q4
    return y.astype(np.float32).reshape(-1)


@pytest.mark.parametrize("qtype", [W.Q5_K, W.Q6_K])
def test_dequantize_matches_ggml_loops(orc, qtype):
    rows, k = 24, 1024
    w = W.weights(qtype, rows, k, seed=qtype)
    got = orc.dequantize(qtype, w, rows, k).ravel()
    assert np.array_equal(got.view(np.uint32), numpy_dequant(qtype, w).view(np.uint32))


@pytest.mark.parametrize("qtype", [W.Q5_K, W.Q6_K])
def test_q81_within_tolerance_of_exact(orc, qtype):
    rows, k = 16, 4096
    w = orc.random_rows(qtype, k, rows, seed=3 + qtype)
    x = np.random.default_rng(qtype).standard_normal(k).astype(np.float32)
    acts = orc.prepare(x)
    rb = w.size // rows
    for r in range(rows):
        e = orc.evaluate(qtype, w[r * rb:(r + 1) * rb], x, acts)
        assert abs(e["q81"] - e["exact"]) <= QMV_NORM_TOL * e["weight_norm"] * np.linalg.norm(x)
        assert np.isnan(e["h16"])   # no h16 model for these formats
    with pytest.raises(ValueError):
        orc.qmv_h16(qtype, w, rows, k, acts, 1, 16)


def test_block_sizes(orc):
    assert [orc.lib.p100o_block_elems(t) for t in range(5)] == [32, 32, 256, 256, 256]
    assert [orc.lib.p100o_block_bytes(t) for t in range(5)] == [18, 34, 144, 176, 210]
