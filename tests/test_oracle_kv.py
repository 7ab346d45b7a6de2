"""The quantised K/V cache oracle (oracle/kv_oracle.cpp) on CPU.

Conversion to fp16 is checked against an independent numpy restatement of
dequantize_q8_0 / dequantize_q4_0 and dequantize_block's view geometry
(bench/micro/dequant_nc.cu:32-77), on blocks drawn by the reference's own
generator (:144-149, itself restated here in plain Python for the first
blocks), in the reference's layout: a token-major K/V view with row stride
n_head_kv * D values and head stride D values (:12-13, :156)."""
import numpy as np
import pytest

import oracle

KV_TYPES = [oracle.KV_Q8_0, oracle.KV_Q4_0]
# The reference's four shapes (dequant_nc.cu:209-214), n_kv cut so numpy stays quick.
SHAPES = [(64, 7680 // 8, 8), (128, 16384 // 16, 8), (256, 16384 // 16, 2), (256, 32768 // 32, 4)]


def blocks_view(raw, kv_type):
    """Raw bytes -> (d float32, codes int [nblk, 32]) by the block layout alone."""
    bb = oracle.KV_BLOCK_BYTES[kv_type]
    b = raw.reshape(-1, bb)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    if kv_type == oracle.KV_Q8_0:
        q = b[:, 2:].view(np.int8).astype(np.float32)
    else:
        qs = b[:, 2:].astype(np.int32)
        q = np.concatenate([qs & 15, qs >> 4], axis=1).astype(np.float32) - 8.0
    return d, q


def numpy_to_f16(raw, kv_type, ne00, ne01, ne02, ne03, s01, s02, s03):
    d, q = blocks_view(raw, kv_type)
    vals = (q * d[:, None]).astype(np.float16)          # exact FP32 product, one rounding
    nb = ne00 // 32
    i03, i02, i01, ib = np.meshgrid(np.arange(ne03), np.arange(ne02), np.arange(ne01), np.arange(nb),
                                    indexing="ij")
    idx = i03 * s03 + i02 * s02 + i01 * s01 + ib
    return vals[idx.ravel()].reshape(ne03, ne02, ne01, ne00)


def test_lcg_matches_a_python_restatement(orc):
    for kv_type in KV_TYPES:
        bb = oracle.KV_BLOCK_BYTES[kv_type]
        raw = orc.kv_lcg_blocks(kv_type, 5)
        r = 12345
        expect = []
        for _ in range(5):
            r = (r * 1664525 + 1013904223) & 0xFFFFFFFF
            d = np.float32(np.float32(0.01) + np.float32(r >> 8) * np.float32(1e-9))
            expect += list(np.array([d], np.float16).view(np.uint8))
            for _ in range(bb - 2):
                r = (r * 1664525 + 1013904223) & 0xFFFFFFFF
                expect.append(r >> 24)
        assert raw.tolist() == [int(x) for x in expect]


@pytest.mark.parametrize("kv_type", KV_TYPES)
@pytest.mark.parametrize("d,n_kv,nh", SHAPES)
def test_to_f16_reference_view(orc, kv_type, d, n_kv, nh):
    nb = d // 32
    raw = orc.kv_lcg_blocks(kv_type, nb * nh * n_kv)
    # token-major cache: row (token) stride nh * nb blocks, head stride nb
    args = (d, n_kv, nh, 1, nb * nh, nb, nb * nh * n_kv)
    got = orc.kv_to_f16(kv_type, raw, *args)
    want = numpy_to_f16(raw, kv_type, *args)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("kv_type", KV_TYPES)
def test_to_f16_subnormal_and_signed_zero(orc, kv_type):
    bb = oracle.KV_BLOCK_BYTES[kv_type]
    rng = np.random.default_rng(3)
    raw = rng.integers(0, 256, size=64 * bb, dtype=np.uint8).reshape(64, bb)
    d = np.array([1e-7, 3e-6, -2e-5, 0.0, -0.0, 6e-5, 1.0, -65000.0 / 128] * 8, dtype=np.float16)
    raw[:, :2] = d.view(np.uint8).reshape(64, 2)
    got = orc.kv_to_f16(kv_type, raw.ravel(), 64, 32)
    want = numpy_to_f16(raw.ravel(), kv_type, 64, 32, 1, 1, 2, 64, 64)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def numpy_quantize(kv_type, x):
    """ggml's quantize_row_q8_0_ref / quantize_row_q4_0_ref restated in numpy."""
    x = x.reshape(-1, 32).astype(np.float32)
    out = []
    for blk in x:
        if kv_type == oracle.KV_Q8_0:
            d = np.float32(np.abs(blk).max()) / np.float32(127)
            idv = np.float32(1) / d if d else np.float32(0)
            q = np.round(blk * idv)                   # ties: see the away-from-zero fix below
            half = np.abs(blk * idv - np.trunc(blk * idv)) == 0.5
            q[half] = np.trunc(blk * idv)[half] + np.sign(blk * idv)[half]
            out.append(np.concatenate([np.array([d], np.float16).view(np.uint8), q.astype(np.int8).view(np.uint8)]))
        else:
            j = int(np.argmax(np.abs(blk)))
            vmax = blk[j] if np.abs(blk[j]) > 0 else np.float32(0)
            d = np.float32(vmax) / np.float32(-8)
            idv = np.float32(1) / d if d else np.float32(0)
            q = np.minimum(15, np.trunc(blk * idv + np.float32(8.5)).astype(np.int32))
            qs = (q[:16] | (q[16:] << 4)).astype(np.uint8)
            out.append(np.concatenate([np.array([d], np.float16).view(np.uint8), qs]))
    return np.concatenate(out)


@pytest.mark.parametrize("kv_type", KV_TYPES)
def test_quantize_matches_numpy_and_round_trips(orc, kv_type):
    rng = np.random.default_rng(kv_type)
    x = (rng.standard_normal(32 * 200) * 0.7).astype(np.float32)
    x[:32] = 0.0                       # all-zero block: d = 0, codes 0 (q8_0) / 8 (q4_0)
    x[32:64] = -0.0
    x[64:96] = np.linspace(-1, 1, 32)  # exact ties of |x| at both ends: the first wins (q4_0)
    raw = orc.kv_quantize(kv_type, x)
    assert np.array_equal(raw, numpy_quantize(kv_type, x))
    back = orc.kv_to_f16(kv_type, raw, 32, x.size // 32).astype(np.float32).ravel()
    d, _ = blocks_view(raw, kv_type)
    step = np.repeat(np.abs(d), 32)
    # q8_0 rounds to the nearest code; q4_0 truncates x/d + 8.5, i.e. rounds
    # too, except that code 16 (x near -vmax) is clamped to 15: one full step
    err = np.abs(back - x)
    slack = np.abs(x) * 2e-3 + 1e-6      # the fp16 rounding of d and of the output
    if kv_type == oracle.KV_Q8_0:
        assert np.all(err <= step * 0.5 + slack)
    else:
        assert np.all(err <= step + slack) and np.mean(err <= step * 0.5 + slack) > 0.95
