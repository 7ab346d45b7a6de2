"""The CPU restatement of the decode-step glue (oracle/decode_oracle.cpp)
checked against plain float64 numpy of the same formulas, and a whole
restated decode step on a tiny model.  The reference has no decode step, so
these are the checks that hold the restatement to the Llama-3 math; the GPU
kernels are then held to the restatement bit for bit (test_decode_gpu.py)."""
import numpy as np
import pytest

import oracle


def test_dec_exp_error_bound(orc):
    """exp by Cody-Waite + Taylor: within 2 ulp of the float64 exponential
    over the normal range, 0 below -104, +inf above 89."""
    xs = np.concatenate([np.linspace(-87.0, 88.0, 200001, dtype=np.float32),
                         np.float32([0.0, -0.0, 1e-8, -1e-8, 0.5, -0.5])])
    got = np.array([orc.dec_exp(float(x)) for x in xs], dtype=np.float64)
    want = np.exp(xs.astype(np.float64))
    ulp = np.spacing(want.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got - want) / ulp) <= 2.0
    assert orc.dec_exp(-105.0) == 0.0 and np.isinf(orc.dec_exp(90.0))
    sub = np.float32(-95.0)   # subnormal result: still close in absolute terms
    assert abs(orc.dec_exp(float(sub)) - np.exp(np.float64(sub))) < 1e-44


@pytest.mark.parametrize("k", [32, 256, 4096, 8192])
def test_rmsnorm_matches_float64(orc, k):
    rng = np.random.default_rng(k)
    x = rng.standard_normal(k).astype(np.float32)
    delta = (0.1 * rng.standard_normal(k)).astype(np.float32)
    w = rng.uniform(0.9, 1.1, k).astype(np.float32)
    xs, q, y = orc.rmsnorm_q8_1(x, w, 1e-5, delta=delta)
    assert np.array_equal(xs, (x + delta).astype(np.float32))
    x64 = xs.astype(np.float64)
    want = x64 / np.sqrt((x64 ** 2).mean() + 1e-5) * w
    assert np.max(np.abs(y - want)) <= 4e-7 * np.max(np.abs(want))
    # the Q8_1 bytes are prepare() of y (the pinned quantiser)
    assert np.array_equal(q, orc.quantize_q8_1(y.reshape(1, k), k))


def test_swiglu_matches_float64(orc):
    rng = np.random.default_rng(3)
    n = 14336
    gu = (3 * rng.standard_normal(2 * n)).astype(np.float32)
    gu[:4] = [0.0, -80.0, 80.0, -20.0]
    q = orc.swiglu_q8_1(gu, n)
    g, u = gu[:n].astype(np.float64), gu[n:].astype(np.float64)
    h = g / (1 + np.exp(-g)) * u
    acts = orc.prepare(h.astype(np.float32))
    # same blocks as quantising the float64 result rounded to float32, except
    # where a code sits within a rounding step of a half-way point
    got = q.reshape(-1, 36)
    want = orc.pack_q8_1(acts).reshape(-1, 36)
    differ = np.nonzero(np.any(got != want, axis=1))[0]
    assert differ.size <= n // 32 // 100


def test_rope_and_append(orc):
    nq, nkv, hd, max_pos, pos = 4, 2, 64, 16, 9
    rng = np.random.default_rng(5)
    qkv = rng.standard_normal((nq + 2 * nkv) * hd).astype(np.float32)
    import p100_b200 as P
    cs = P.rope_table(max_pos, hd, 500000.0)
    stride = max_pos * hd
    kc = np.zeros(nkv * stride, dtype=np.uint16)
    vc = np.zeros(nkv * stride, dtype=np.uint16)
    out = orc.rope_kv_append(qkv, nq, nkv, hd, cs, max_pos, pos, kc, vc, stride)
    ang = pos * 500000.0 ** (-2.0 * np.arange(hd // 2) / hd)
    c, s = np.cos(ang), np.sin(ang)
    for h in range(nq):
        x = qkv[h * hd:(h + 1) * hd].astype(np.float64)
        want = np.empty(hd)
        want[0::2] = x[0::2] * c - x[1::2] * s
        want[1::2] = x[0::2] * s + x[1::2] * c
        assert np.max(np.abs(out[h * hd:(h + 1) * hd] - want)) < 1e-5
    # v rows are the fp16 values, other rows untouched
    for h in range(nkv):
        v = qkv[(nq + nkv + h) * hd:(nq + nkv + h + 1) * hd]
        row = vc[h * stride + pos * hd:h * stride + (pos + 1) * hd]
        assert np.array_equal(row, v.astype(np.float16).view(np.uint16))
    assert np.count_nonzero(vc) == np.count_nonzero(vc[[h * stride + pos * hd + e for h in range(nkv)
                                                         for e in range(hd)]])


def test_argmax_ties_and_nan(orc):
    assert orc.argmax(np.float32([1, 5, 5, 2]))[0] == 1
    assert orc.argmax(np.float32([np.nan, 1, np.nan, 3]))[0] == 3
    assert orc.argmax(np.float32([np.nan, np.nan]))[0] == 0
    assert orc.argmax(np.float32([-np.inf, -np.inf]))[0] == 0


def tiny_model(orc, wtype=oracle.Q4_0, seed=11):
    cfg = oracle.LlamaConfig(2, 256, 4, 2, 64, 512, 300, 32, 500000.0, 1e-5, wtype)
    rng = np.random.default_rng(seed)
    rows = lambda r, k, s: orc.random_rows(wtype, k, r, s)   # noqa: E731
    hd = cfg.head_dim
    w = {"embed": rows(cfg.vocab, cfg.hidden, seed), "out_norm": rng.uniform(0.9, 1.1, cfg.hidden).astype(np.float32),
         "lm_head": rows(cfg.vocab, cfg.hidden, seed + 1)}
    for name in ("attn_norm", "ffn_norm", "wqkv", "wo", "wgu", "wdown"):
        w[name] = []
    for l in range(cfg.n_layer):
        w["attn_norm"].append(rng.uniform(0.9, 1.1, cfg.hidden).astype(np.float32))
        w["ffn_norm"].append(rng.uniform(0.9, 1.1, cfg.hidden).astype(np.float32))
        w["wqkv"].append(rows((cfg.n_head + 2 * cfg.n_head_kv) * hd, cfg.hidden, seed + 10 + l))
        w["wo"].append(rows(cfg.hidden, cfg.n_head * hd, seed + 20 + l))
        w["wgu"].append(rows(2 * cfg.ffn, cfg.hidden, seed + 30 + l))
        w["wdown"].append(rows(cfg.hidden, cfg.ffn, seed + 40 + l))
    return cfg, w


def test_decode_step_runs_and_is_deterministic(orc):
    import p100_b200 as P
    cfg, w = tiny_model(orc)
    cs = P.rope_table(cfg.max_ctx, cfg.head_dim, cfg.rope_theta)
    n = cfg.n_layer * cfg.n_head_kv * cfg.max_ctx * cfg.head_dim
    outs = []
    for _ in range(2):
        kc = np.zeros(n, dtype=np.uint16)
        vc = np.zeros(n, dtype=np.uint16)
        toks, tok = [], 3
        for pos in range(4):
            tok, logits, hidden = orc.decode_step(cfg, w, kc, vc, cs, pos, tok)
            assert np.all(np.isfinite(logits)) and 0 <= tok < cfg.vocab
            assert tok == int(np.argmax(logits))
            toks.append(tok)
        outs.append((toks, logits.copy(), kc.copy()))
    assert outs[0][0] == outs[1][0]
    assert np.array_equal(outs[0][1], outs[1][1]) and np.array_equal(outs[0][2], outs[1][2])
    # the cache holds rows 0..3 of every layer and head, nothing beyond
    kc4 = outs[0][2].reshape(cfg.n_layer, cfg.n_head_kv, cfg.max_ctx, cfg.head_dim)
    assert np.count_nonzero(kc4[:, :, :4]) > 0 and np.count_nonzero(kc4[:, :, 4:]) == 0
