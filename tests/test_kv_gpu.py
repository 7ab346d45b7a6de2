"""Quantised K/V cache on B200: p100_kv_to_f16 and FlashAttention decode over
q8_0 / q4_0 K/V (C-ABI), against the CPU restatement in oracle/kv_oracle.cpp.

Bars: the conversion is bit-exact (each value is one rounding of an exact
product, dequant_nc.cu:32-48).  The decode over a quantised cache equals the
fp16 decode over the converted cache bit for bit (the kernel dequantises the
same values into the same tiles), and meets the attention tolerance against
attention_reference on the dequantised K/V."""
import numpy as np
import pytest

from conftest import ATTN_MAX_REL_TOL, lse_within_tolerance, out_within_tolerance

import oracle
import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu
KV_TYPES = [P.KV_Q8_0, P.KV_Q4_0]
# The reference's shapes (bench/micro/dequant_nc.cu:209-214): D, n_kv, n_head_kv.
REF_SHAPES = [(64, 7680, 8), (128, 16384, 8), (256, 16384, 2), (256, 32768, 4)]


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("d,n_kv,nh", REF_SHAPES)
def test_to_f16_reference_shapes(cuda, orc, kv_type, d, n_kv, nh):
    """The reference's view (token-major rows of n_head_kv * D values, heads D
    apart) over its own LCG blocks, at full size."""
    nb = d // 32
    raw = orc.kv_lcg_blocks(kv_type, nb * nh * n_kv)
    args = (d, n_kv, nh, 1, nb * nh, nb, nb * nh * n_kv)
    got = P.kv_to_f16(kv_type, dev(cuda, raw), *args).cpu().numpy()
    want = orc.kv_to_f16(kv_type, raw, *args)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("kv_type", KV_TYPES)
def test_to_f16_odd_views_and_tiny_scales(cuda, orc, kv_type):
    """A 4-d view with gaps between rows and planes, an odd block offset (the
    source only 2-byte aligned), random bytes with subnormal and signed-zero
    scales."""
    bb = P.KV_BLOCK_BYTES[kv_type]
    ne00, ne01, ne02, ne03 = 96, 37, 3, 2
    s01, s02, s03 = 5, 5 * 40, 5 * 40 * 3 + 7
    nblk = s03 * ne03 + 1
    rng = np.random.default_rng(kv_type)
    raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    d = rng.choice(np.array([1e-7, 2e-6, -3e-5, 0.0, -0.0, 0.01, -0.7, 3.0], np.float16), size=nblk)
    raw[:, :2] = d.view(np.uint8).reshape(nblk, 2)
    src = dev(cuda, raw.ravel())[bb:]      # start one block in: 2-byte aligned only
    got = P.kv_to_f16(kv_type, src, ne00, ne01, ne02, ne03, s01, s02, s03).cpu().numpy()
    want = orc.kv_to_f16(kv_type, raw.ravel()[bb:], ne00, ne01, ne02, ne03, s01, s02, s03)
    assert np.array_equal(bits(got), bits(want))


def quantised_cache(orc, kv_type, k, cap=None):
    """[B,H,S,D] values -> uint8 [B,H,cap,D/32*bb] blocks (rows past S zero)."""
    b, h, s, d = k.shape
    cap = cap or s
    rb = d // 32 * P.KV_BLOCK_BYTES[kv_type]
    out = np.zeros((b, h, cap, rb), np.uint8)
    out[:, :, :s] = orc.kv_quantize(kv_type, k.astype(np.float32)).reshape(b, h, s, rb)
    return out


def check_attention(o, lse, ref_o, ref_lse):
    o, lse = o.astype(np.float64), lse.astype(np.float64)
    assert out_within_tolerance(o, ref_o).all(), f"max abs err {np.abs(o - ref_o).max():.3e}"
    assert lse_within_tolerance(lse, ref_lse).all()
    if np.abs(ref_o).max() > 0:
        assert np.abs(o - ref_o).max() / np.abs(ref_o).max() <= ATTN_MAX_REL_TOL


def run_pair(cuda, orc, kv_type, batch, hq, hkv, seq, d, splits=0, cap=None, seed=0):
    """Quantised decode vs fp16 decode of the converted cache (bit for bit);
    returns the outputs and the dequantised K/V for a reference check."""
    q, k, v = W.attention_inputs(batch, hq, hkv, seq, d, seed=seed)
    cap = cap or seq
    kq, vq = quantised_cache(orc, kv_type, k, cap), quantised_cache(orc, kv_type, v, cap)
    nb = d // 32
    desc = P.AttnDesc(batch=batch, n_head_q=hq, n_head_kv=hkv, seq_kv=seq, d_qk=d, d_v=d, kv_splits=splits,
                      kv_head_stride=cap * d, kv_batch_stride=hkv * cap * d, kv_type=kv_type)
    gq, gk, gv = dev(cuda, q), dev(cuda, kq), dev(cuda, vq)
    o, lse = P.fa_decode(desc, gq, gk, gv)
    # the converted cache: rows [0, seq) of every head, contiguous fp16
    conv = dict(ne00=d, ne01=seq, ne02=hkv, ne03=batch, s01=nb, s02=cap * nb, s03=hkv * cap * nb)
    kf = P.kv_to_f16(kv_type, gk, **conv)
    vf = P.kv_to_f16(kv_type, gv, **conv)
    desc16 = P.AttnDesc(batch=batch, n_head_q=hq, n_head_kv=hkv, seq_kv=seq, d_qk=d, d_v=d, kv_splits=splits)
    o16, lse16 = P.fa_decode(desc16, gq, kf, vf)
    assert P.device_error() == P.OK
    return (o.cpu().numpy(), lse.cpu().numpy(), o16.cpu().numpy(), lse16.cpu().numpy(), q,
            kf.cpu().numpy().astype(np.float32), vf.cpu().numpy().astype(np.float32))


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 8), (64, 8)])
def test_decode_equals_converted_fp16(cuda, orc, kv_type, d, hq, hkv):
    o, lse, o16, lse16, q, kf, vf = run_pair(cuda, orc, kv_type, 1, hq, hkv, 1000, d, seed=hq + d)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), lse16.view(np.uint32))
    p = oracle.Attn(n_head_q=hq, n_head_kv=hkv, seq_kv=1000, d_qk=d, d_v=d)
    ref_o, ref_lse = orc.attention_reference(p, q, kf, vf)
    check_attention(o, lse, ref_o, ref_lse)


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("seq", [1, 2, 63, 64, 65, 129, 4096, 16384])
def test_ragged_and_contexts_to_16k(cuda, orc, kv_type, seq):
    """Short tails and the cluster merge (automatic split up to 16K keys, the
    same split as the fp16 decode)."""
    o, lse, o16, lse16, *_ = run_pair(cuda, orc, kv_type, 1, 32, 8, seq, 128, seed=seq)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), lse16.view(np.uint32))


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("seq", [8192, 8193, 20000, 32768])
def test_long_contexts(cuda, orc, kv_type, seq):
    """Past 8K keys the automatic split runs the 8-warp shape (128-key tiles,
    one part per SM, workspace merge) for both caches: bit-exact, and within
    the attention tolerance of attention_reference; at 8192 keys the 4-warp
    cluster merge still runs."""
    o, lse, o16, lse16, q, kf, vf = run_pair(cuda, orc, kv_type, 1, 32, 8, seq, 128, seed=seq)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), lse16.view(np.uint32))
    if seq == 20000:
        p = oracle.Attn(n_head_q=32, n_head_kv=8, seq_kv=seq, d_qk=128, d_v=128)
        ref_o, ref_lse, _ = orc.attention_reference_threaded(p, q, kf, vf, oracle.host_cores())
        check_attention(o, lse, ref_o, ref_lse)


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("hq,hkv,d", [(64, 8, 64), (8, 8, 128), (16, 2, 64)])
def test_long_contexts_other_groups(cuda, orc, kv_type, hq, hkv, d):
    """The 8-warp shape with d 64 and groups of 8, 1 and 8 query heads, batch 2."""
    o, lse, o16, lse16, q, kf, vf = run_pair(cuda, orc, kv_type, 2, hq, hkv, 9000, d, seed=hq + d)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))
    p = oracle.Attn(batch=2, n_head_q=hq, n_head_kv=hkv, seq_kv=9000, d_qk=d, d_v=d)
    ref_o, ref_lse, _ = orc.attention_reference_threaded(p, q, kf, vf, oracle.host_cores())
    check_attention(o, lse, ref_o, ref_lse)


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("splits", [1, 3, 7, 16])
def test_explicit_splits(cuda, orc, kv_type, splits):
    o, lse, o16, lse16, *_ = run_pair(cuda, orc, kv_type, 1, 32, 8, 3001, 128, splits=splits, seed=splits)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("d,cap", [(128, 1001), (64, 777), (64, 1003)])
def test_cache_capacity_unaligned_heads(cuda, orc, kv_type, d, cap):
    """Capacity > seq with odd capacities, so heads (and parts) start off the
    16-byte grid; batch 2; the last head's rows end at the buffer's end."""
    o, lse, o16, lse16, q, kf, vf = run_pair(cuda, orc, kv_type, 2, 16, 4, cap - 3, d, cap=cap, seed=cap)
    assert np.array_equal(o.view(np.uint32), o16.view(np.uint32))
    o2, lse2, o162, *_ = run_pair(cuda, orc, kv_type, 2, 16, 4, cap, d, cap=cap, seed=cap)
    assert np.array_equal(o2.view(np.uint32), o162.view(np.uint32))


def test_rejections(cuda):
    z = cuda.zeros(1 << 16, dtype=cuda.uint8, device="cuda")
    q = cuda.zeros(64 * 256, device="cuda")
    for desc, err in [
        (P.AttnDesc(n_head_q=8, n_head_kv=8, seq_kv=64, d_qk=256, d_v=256, kv_type=P.KV_Q8_0), P.ERR_UNSUPPORTED),
        (P.AttnDesc(n_head_q=24, n_head_kv=8, seq_kv=64, kv_type=P.KV_Q8_0), P.ERR_UNSUPPORTED),   # G = 3
        (P.AttnDesc(n_head_q=8, n_head_kv=8, seq_kv=64, kv_type=P.KV_Q4_0, kv_head_stride=64 * 128 + 32),
         P.ERR_INVALID),
        (P.AttnDesc(n_head_q=8, n_head_kv=8, seq_kv=64, kv_type=5), P.ERR_INVALID),
    ]:
        with pytest.raises(P.P100Error) as e:
            P.fa_decode(desc, q, z, z, ws=z)
        assert e.value.status == err
