"""GPU parity of the split-K FlashAttention-vec decode kernel (C-ABI).

Bar (include/p100/tolerance.h:20-31, tests/error_budget.cpp:78): every output
within 1e-3 + 2e-3*|ref| of attention_reference, LSE within 1e-3, and
max|O - O_ref| / max|O_ref| <= 1e-3; fully masked rows give O = 0, LSE = -inf."""
import numpy as np
import pytest

from conftest import ATTN_MAX_REL_TOL, golden, lse_within_tolerance, out_within_tolerance

import oracle
import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_attention(o, lse, ref_o, ref_lse):
    o, lse = o.astype(np.float64), lse.astype(np.float64)
    assert out_within_tolerance(o, ref_o).all(), f"max abs err {np.abs(o - ref_o).max():.3e}"
    assert lse_within_tolerance(lse, ref_lse).all()
    if np.abs(ref_o).max() > 0:
        assert np.abs(o - ref_o).max() / np.abs(ref_o).max() <= ATTN_MAX_REL_TOL


def run_fa(torch, desc, q, k, v, mask=None):
    o, lse = P.fa_decode(desc, dev(torch, q), dev(torch, k), dev(torch, v),
                         None if mask is None else dev(torch, mask))
    return o.cpu().numpy(), lse.cpu().numpy()


def test_golden_cases(cuda):
    g = golden("attention.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_params")})
    for name in names:
        b, hq, hkv, s, d = (int(x) for x in g[name + "_params"])
        scale, softcap = (float(x) for x in g[name + "_scales"])
        desc = P.AttnDesc(batch=b, n_head_q=hq, n_head_kv=hkv, seq_q=1, seq_kv=s, d_qk=d, d_v=d, scale=scale,
                          softcap=softcap)
        mask = g[name + "_mask"] if name + "_mask" in g.files else None
        o, lse = run_fa(cuda, desc, g[name + "_q"], g[name + "_k"], g[name + "_v"], mask)
        check_attention(o, lse, g[name + "_o"], g[name + "_lse"])
    # the split-K model of the same inputs agrees too
    name = "gqa4_d128_s450"
    b, hq, hkv, s, d = (int(x) for x in g[name + "_params"])
    desc = P.AttnDesc(batch=b, n_head_q=hq, n_head_kv=hkv, seq_kv=s, d_qk=d, d_v=d, kv_splits=4)
    o, lse = run_fa(cuda, desc, g[name + "_q"], g[name + "_k"], g[name + "_v"])
    check_attention(o, lse, g[name + "_split4_o"], g[name + "_split4_lse"])


def test_all_masked_row(cuda):
    g = golden("attention.npz")
    name = "allmasked_d128_s70"
    desc = P.AttnDesc(n_head_q=4, n_head_kv=1, seq_kv=70, kv_splits=1)
    for splits in (1, 0):
        desc.kv_splits = splits
        o, lse = run_fa(cuda, desc, g[name + "_q"], g[name + "_k"], g[name + "_v"], g[name + "_mask"])
        assert np.all(o == 0) and np.all(np.isneginf(lse))


@pytest.mark.parametrize("seq_kv", [512, 4096, 16384, 32768])
def test_config3_shapes(cuda, orc, seq_kv):
    """Config 3: 32 query / 8 KV heads, d=128, the four context lengths."""
    q, k, v = W.attention_inputs(1, 32, 8, seq_kv, 128, seed=seq_kv)
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=seq_kv, d_qk=128, d_v=128)
    o, lse = run_fa(cuda, desc, q, k, v)
    p = oracle.Attn(n_head_q=32, n_head_kv=8, seq_kv=seq_kv, d_qk=128, d_v=128)
    ref_o, ref_lse, _ = orc.attention_reference_threaded(p, q, k.astype(np.float32), v.astype(np.float32),
                                                         oracle.host_cores())
    check_attention(o, lse, ref_o, ref_lse)


@pytest.mark.parametrize("hq,hkv,d", [(64, 8, 128), (8, 8, 128), (16, 8, 128), (12, 4, 128), (28, 4, 128),
                                      (32, 8, 64), (16, 8, 256), (40, 8, 64)])
def test_gqa_and_head_dims(cuda, orc, hq, hkv, d):
    q, k, v = W.attention_inputs(2, hq, hkv, 777, d, seed=hq * d)
    desc = P.AttnDesc(batch=2, n_head_q=hq, n_head_kv=hkv, seq_kv=777, d_qk=d, d_v=d)
    o, lse = run_fa(cuda, desc, q, k, v)
    p = oracle.Attn(batch=2, n_head_q=hq, n_head_kv=hkv, seq_kv=777, d_qk=d, d_v=d)
    ref_o, ref_lse = orc.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32))
    check_attention(o, lse, ref_o, ref_lse)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 16, 0])
def test_split_counts_agree(cuda, orc, splits):
    q, k, v = W.attention_inputs(1, 32, 8, 2000, 128, seed=9)
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=2000, kv_splits=splits)
    o, lse = run_fa(cuda, desc, q, k, v)
    p = oracle.Attn(n_head_q=32, n_head_kv=8, seq_kv=2000)
    ref_o, ref_lse = orc.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32))
    check_attention(o, lse, ref_o, ref_lse)
    # and the FP32 tiled model with the same number of parts
    if splits:
        cfg = oracle.Tiled(1, 64, False, False, False, kv_parallel_blocks=splits)
        t_o, t_lse = orc.attention_tiled(p, cfg, q, k.astype(np.float32), v.astype(np.float32))
        check_attention(o, lse, t_o, t_lse)


@pytest.mark.parametrize("seq_kv", [1, 2, 63, 64, 65, 127, 129, 1000])
def test_ragged_lengths(cuda, orc, seq_kv):
    q, k, v = W.attention_inputs(1, 8, 2, seq_kv, 128, seed=seq_kv + 1)
    desc = P.AttnDesc(n_head_q=8, n_head_kv=2, seq_kv=seq_kv)
    o, lse = run_fa(cuda, desc, q, k, v)
    p = oracle.Attn(n_head_q=8, n_head_kv=2, seq_kv=seq_kv)
    ref_o, ref_lse = orc.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32))
    check_attention(o, lse, ref_o, ref_lse)


def test_kv_cache_strides(cuda, orc):
    """A cache with capacity 1024 holding 700 keys gives the contiguous result."""
    q, k, v = W.attention_inputs(2, 16, 4, 700, 128, seed=4)
    cap = 1024
    kc = np.zeros((2, 4, cap, 128), np.float16)
    vc = np.zeros_like(kc)
    kc[:, :, :700], vc[:, :, :700] = k, v
    desc = P.AttnDesc(batch=2, n_head_q=16, n_head_kv=4, seq_kv=700, kv_head_stride=cap * 128,
                      kv_batch_stride=4 * cap * 128)
    o, lse = run_fa(cuda, desc, q, kc, vc)
    p = oracle.Attn(batch=2, n_head_q=16, n_head_kv=4, seq_kv=700)
    ref_o, ref_lse = orc.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32))
    check_attention(o, lse, ref_o, ref_lse)


def test_softcap_and_scale(cuda, orc):
    q, k, v = W.attention_inputs(1, 8, 2, 300, 128, seed=11)
    desc = P.AttnDesc(n_head_q=8, n_head_kv=2, seq_kv=300, scale=0.3, softcap=20.0)
    o, lse = run_fa(cuda, desc, q, k, v)
    p = oracle.Attn(n_head_q=8, n_head_kv=2, seq_kv=300, scale=0.3, softcap=20.0)
    ref_o, ref_lse = orc.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32))
    check_attention(o, lse, ref_o, ref_lse)


def test_workspace_reuse_is_deterministic(cuda):
    q, k, v = W.attention_inputs(1, 32, 8, 4096, 128, seed=12)
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=4096)
    ws = P.fa_workspace(desc)
    qd, kd, vd = dev(cuda, q), dev(cuda, k), dev(cuda, v)
    first = [t.clone() for t in P.fa_decode(desc, qd, kd, vd, ws=ws)]
    for _ in range(4):
        o, lse = P.fa_decode(desc, qd, kd, vd, ws=ws)
        assert cuda.equal(o, first[0]) and cuda.equal(lse, first[1])
    assert P.device_error() == P.OK


def test_invalid_descriptors(cuda):
    q = cuda.zeros(4096, device="cuda")
    kv = cuda.zeros(4096, dtype=cuda.float16, device="cuda")
    with pytest.raises(P.InvalidArgument, match="n_head_q must be divisible by n_head_kv"):
        P.fa_decode(P.AttnDesc(n_head_q=3, n_head_kv=2), q, kv, kv, ws=None)
    with pytest.raises(P.InvalidArgument, match="all dimensions must be positive"):
        P.fa_decode(P.AttnDesc(seq_kv=0), q, kv, kv, ws=None)
    with pytest.raises(P.P100Error) as err:
        P.fa_decode(P.AttnDesc(seq_q=2, seq_kv=8), q, kv, kv, ws=None)
    assert err.value.status == P.ERR_UNSUPPORTED
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=4096)
    with pytest.raises(P.InvalidArgument, match="workspace"):
        small = cuda.zeros(16, dtype=cuda.uint8, device="cuda")
        P.fa_decode(desc, cuda.zeros(32 * 128, device="cuda"), cuda.zeros(8 * 4096 * 128, dtype=cuda.float16,
                    device="cuda"), cuda.zeros(8 * 4096 * 128, dtype=cuda.float16, device="cuda"), ws=small)
