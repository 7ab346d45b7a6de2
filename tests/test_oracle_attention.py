"""The oracle's attention contract on CPU: the reference's analytic cases
(tests/test_reference.cpp:22-201), its tiled-model pins (the FNV digest of
tests/test_tiled_model_flush.cpp:43-66 and the consistency line of
tests/error_budget_split.cpp:122-136), the golden fixtures, and agreement with
the reference library itself."""
import math

import numpy as np
import pytest

from conftest import golden, lse_within_tolerance, out_within_tolerance

import oracle

INF = float("inf")


def small(nq, nk, dq, dv, **kw):
    kw.setdefault("scale", 1.0)
    return oracle.Attn(seq_q=nq, seq_kv=nk, d_qk=dq, d_v=dv, **kw)


def arr(*v):
    return np.array(v, np.float32)


def test_tiny(orc):
    p = small(2, 2, 2, 2)
    o, lse = orc.attention_reference(p, arr(1, 0, 0, 1), arr(math.log(3), 0, 0, math.log(3)), arr(2, 4, 6, 8))
    assert np.allclose(o.ravel(), [3, 5, 5, 7], atol=1e-6)
    assert np.allclose(lse.ravel(), math.log(4), atol=1e-6)


def test_uniform_and_default_scale(orc):
    p = small(2, 3, 2, 3, scale=0.0)
    assert abs(orc.effective_scale(p) - 1 / math.sqrt(2)) < 1e-7
    o, lse = orc.attention_reference(p, np.zeros(4, np.float32), arr(1, 2, 3, 4, 5, 6),
                                     arr(1, 2, 6, 3, 4, 0, 8, 9, -3))
    assert np.array_equal(o.reshape(2, 3), [[4, 5, 1], [4, 5, 1]])
    assert np.allclose(lse, math.log(3), atol=1e-7)


def test_gqa_head_mapping(orc):
    p = small(2, 3, 1, 2, batch=2, n_head_q=8, n_head_kv=2)
    v = np.zeros((2, 2, 3, 2), np.float32)
    for b in range(2):
        for h in range(2):
            for j in range(3):
                v[b, h, j] = [100 * b + 10 * h + j, -(100 * b + 10 * h + j)]
    o, _ = orc.attention_reference(p, np.zeros(32, np.float32), np.zeros(12, np.float32), v)
    for b in range(2):
        for h in range(8):
            e = 100 * b + 10 * (h // 4) + 1
            assert np.all(o[b, h, :, 0] == e) and np.all(o[b, h, :, 1] == -e)


def test_double_accumulation(orc):
    o, _ = orc.attention_reference(small(1, 2, 3, 1), arr(1, 1, 1), arr(1e8, 1, -1e8, 0, 0, 0), arr(0, 1))
    assert abs(o.item() - 1 / (1 + math.e)) < 1e-7
    o, _ = orc.attention_reference(small(1, 3, 1, 1), arr(0), arr(0, 0, 0), arr(1e8, 1, -1e8))
    assert abs(o.item() - 1 / 3) < 1e-7


def test_causal_bottom_right(orc):
    p = small(3, 5, 1, 1, causal=True)
    o, lse = orc.attention_reference(p, arr(0, 0, 0), arr(0, 0, 0, 0, 0), arr(0, 2, 4, 6, 8))
    assert np.array_equal(o.ravel(), [2, 3, 4])
    assert np.allclose(lse.ravel(), np.log([3, 4, 5]), atol=1e-7)
    p = small(5, 3, 1, 1, causal=True)
    o, lse = orc.attention_reference(p, arr(0, 0, 0), arr(0, 0, 0, 0, 0), arr(0, 2, 4))
    assert np.array_equal(o.ravel()[:2], [0, 0]) and np.all(np.isneginf(lse.ravel()[:2]))
    assert np.array_equal(o.ravel()[2:], [0, 1, 2])


def test_masked_rows(orc):
    p = small(2, 3, 1, 2)
    mask = arr(-INF, -INF, -INF, -INF, 0, -INF)
    o, lse = orc.attention_reference(p, arr(1, 1), arr(1, 2, 3), arr(1, 2, 3, 4, 5, 6), mask)
    assert np.array_equal(o.ravel(), [0, 0, 3, 4]) and np.isneginf(lse.ravel()[0]) and lse.ravel()[1] == 2


def test_softcap(orc):
    p = small(1, 2, 1, 1, scale=2.0, softcap=3.0)
    o, lse = orc.attention_reference(p, arr(10), arr(10, -10), arr(2, 9), arr(-4, 1))
    a, b = 3 * math.tanh(200 / 3) - 4, 3 * math.tanh(-200 / 3) + 1
    s = math.exp(a) + math.exp(b)
    assert abs(o.item() - (2 * math.exp(a) + 9 * math.exp(b)) / s) < 1e-6
    assert abs(lse.item() - math.log(s)) < 1e-7


def test_large_logits(orc):
    o, lse = orc.attention_reference(small(1, 3, 1, 2, scale=10000), arr(1), arr(-1, 1, 0), arr(1, 2, 7, -3, 9, 10))
    assert np.array_equal(o.ravel(), [7, -3]) and lse.item() == 10000


VALIDATION = [
    (dict(batch=0), "all dimensions must be positive"),
    (dict(n_head_q=-1), "all dimensions must be positive"),
    (dict(seq_kv=0), "all dimensions must be positive"),
    (dict(d_v=-1), "all dimensions must be positive"),
    (dict(n_head_q=3, n_head_kv=2), "n_head_q must be divisible by n_head_kv"),
    (dict(softcap=-1.0), "softcap must be finite and non-negative"),
    (dict(softcap=INF), "softcap must be finite and non-negative"),
    (dict(scale=float("nan")), "scale must be finite"),
    (dict(scale=-INF), "scale must be finite"),
]


@pytest.mark.parametrize("kw,why", VALIDATION)
def test_validation_reasons(orc, kw, why):
    ok, reason = orc.validate(oracle.Attn(**kw))
    assert not ok and reason == why
    # rejected before any buffer is touched (null pointers, as test_reference.cpp:158)
    import ctypes
    assert orc._attn_ref(ctypes.byref(oracle.Attn(**kw)), None, None, None, None, None, None) == -1
    assert orc.last_error() == why


def test_validation_accepts(orc):
    assert orc.validate(oracle.Attn(seq_q=5, seq_kv=3, causal=True)) == (True, "")
    p = oracle.Attn(scale=-2.0)
    assert orc.validate(p)[0] and orc.effective_scale(p) == -2.0


# ------------------------------------------------------------- tiled model pins
def test_flush_digest(orc):
    """tests/test_tiled_model_flush.cpp:43-66: FNV-1a over the pre-flush model."""
    p = oracle.Attn(seq_q=3, seq_kv=137, d_qk=64, d_v=64)
    n = 3 * 64 + 2 * 137 * 64
    vals = orc.fill_uniform(20261010, n, -1.0, 1.0, round_fp16=True)
    q, k, v = vals[:192], vals[192:192 + 137 * 64], vals[192 + 137 * 64:]
    cfg = oracle.Tiled(2, 16, False, True, False, o_accum_fp16=1, kv_parallel_blocks=3, o_accum_np=4,
                       kq_max_offset=3 * 0.6931, l_from_unrounded_p=1)
    o, lse = orc.attention_tiled(p, cfg, q, k, v)
    h = 14695981039346656037
    for x in np.concatenate([o.ravel(), lse.ravel()]).view(np.uint32):
        h = ((h ^ int(x)) * 1099511628211) & (2 ** 64 - 1)
    assert h == 12704262495437203684


def _metrics(ref_o, ref_lse, o, lse):
    err = np.abs(o.astype(np.float64) - ref_o)
    max_abs = err.max()
    return (max_abs, max_abs / np.abs(ref_o).max(), err.mean(), np.abs(lse.astype(np.float64) - ref_lse).max())


def test_split_consistency_line(orc):
    """tests/error_budget_split.cpp:122-136: L60 config, d=128, 4096 keys."""
    d, nk, sq = 128, 4096, 16
    vals = orc.fill_normal(12345 + d * 100 + nk, sq * d + 2 * nk * d, round_fp16=True)
    q, k, v = vals[:sq * d], vals[sq * d:sq * d + nk * d], vals[sq * d + nk * d:]
    p = oracle.Attn(seq_q=sq, seq_kv=nk, d_qk=d, d_v=d)
    ref_o, ref_lse = orc.attention_reference(p, q, k, v)
    cfg = oracle.Tiled(32, 64, False, True, True, qk_scale_in_q=1, qk_q_prescale=0.25, qk_products_fp16=1,
                       kq_max_offset=3 * 0.6931, l_from_unrounded_p=1, o_accum_fp16=1)
    o, lse = orc.attention_tiled(p, cfg, q, k, v)
    m = _metrics(ref_o, ref_lse, o, lse)
    line = "L60 normal 128 4096 0 " + " ".join(f"{x:.6e}" for x in m) + " 0"
    assert line == "L60 normal 128 4096 0 1.232397e-03 1.425396e-02 1.567871e-04 6.484985e-05 0"


def test_split_fp32_equivalence(orc):
    """tests/test_tiled_model_split.cpp:14-39: 4 parts/4 accumulators == 1/1."""
    p = oracle.Attn(batch=2, n_head_q=4, n_head_kv=2, seq_q=7, seq_kv=137, d_qk=64, d_v=33)
    rng = np.random.default_rng(5)
    qs, ks, vs, _, _ = p.shapes()
    q, k, v = (rng.uniform(-1, 1, s).astype(np.float32) for s in (qs, ks, vs))
    mask = np.zeros((7, 137), np.float32)
    mask[0] = -INF
    mask[1, 1:] = -INF
    for causal in (False, True):
        p.causal = int(causal)
        base, base_lse = orc.attention_tiled(p, oracle.Tiled(3, 16, False, False, False), q, k, v, mask)
        out, lse = orc.attention_tiled(p, oracle.Tiled(3, 16, False, False, False, kv_parallel_blocks=4,
                                                       o_accum_np=4), q, k, v, mask)
        assert out_within_tolerance(out, base).all() and lse_within_tolerance(lse, base_lse).all()


def test_golden_attention(orc):
    g = golden("attention.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_params")})
    for name in names:
        b, hq, hkv, s, d = (int(x) for x in g[name + "_params"])
        scale, softcap = (float(x) for x in g[name + "_scales"])
        p = oracle.Attn(batch=b, n_head_q=hq, n_head_kv=hkv, seq_q=1, seq_kv=s, d_qk=d, d_v=d, scale=scale,
                        softcap=softcap)
        mask = g[name + "_mask"] if name + "_mask" in g.files else None
        o, lse = orc.attention_reference(p, g[name + "_q"], g[name + "_k"].astype(np.float32),
                                         g[name + "_v"].astype(np.float32), mask)
        assert o.tobytes() == g[name + "_o"].tobytes(), name
        assert lse.tobytes() == g[name + "_lse"].tobytes(), name
    name = "gqa4_d128_s450"
    b, hq, hkv, s, d = (int(x) for x in g[name + "_params"])
    p = oracle.Attn(batch=b, n_head_q=hq, n_head_kv=hkv, seq_q=1, seq_kv=s, d_qk=d, d_v=d)
    o, lse = orc.attention_tiled(p, oracle.Tiled(1, 64, False, False, False, kv_parallel_blocks=4),
                                 g[name + "_q"], g[name + "_k"].astype(np.float32), g[name + "_v"].astype(np.float32))
    assert o.tobytes() == g[name + "_split4_o"].tobytes() and lse.tobytes() == g[name + "_split4_lse"].tobytes()


# ------------------------------------------------------------- against oracle/_ref
def test_reference_and_tiled_match_reference_library(orc, ref):
    rng = np.random.default_rng(21)
    configs = [oracle.Tiled(16, 16, False, False, False), oracle.Tiled(32, 64, True, True, True),
               oracle.Tiled(7, 33, False, True, False, kv_parallel_blocks=3, o_accum_np=2),
               oracle.Tiled(32, 64, False, True, True, qk_half2_chain=4, qk_scale_in_q=1, qk_q_prescale=0.25),
               oracle.Tiled(32, 64, False, True, True, qk_products_fp16=1, o_accum_fp16=1,
                            o_accum_fp16_tile_flush=1, kv_parallel_blocks=2, o_accum_np=4)]
    for trial in range(4):
        p = oracle.Attn(batch=1 + trial % 2, n_head_q=4, n_head_kv=2 - trial % 2, seq_q=1 + 3 * trial,
                        seq_kv=20 + 37 * trial, d_qk=16 * (1 + trial), d_v=16 * (1 + trial) - trial,
                        causal=trial % 2 == 1, softcap=5.0 if trial == 3 else 0.0)
        qs, ks, vs, _, _ = p.shapes()
        q, k, v = (rng.standard_normal(s).astype(np.float32) for s in (qs, ks, vs))
        mask = np.where(rng.random((p.seq_q, p.seq_kv)) < 0.2, -INF, 0).astype(np.float32) if trial == 2 else None
        a = orc.attention_reference(p, q, k, v, mask)
        b = ref.attention_reference(p, q, k, v, mask)
        assert a[0].tobytes() == b[0].tobytes() and a[1].tobytes() == b[1].tobytes()
        for cfg in configs:
            a = orc.attention_tiled(p, cfg, q, k, v, mask)
            b = ref.attention_tiled(p, cfg, q, k, v, mask)
            assert a[0].tobytes() == b[0].tobytes() and a[1].tobytes() == b[1].tobytes()
