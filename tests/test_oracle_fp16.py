"""The oracle's binary16 rounding: known patterns, exhaustive halves and ties,
and agreement with the reference's own round_to_fp16 (CPU only).

Restates the checks of the reference's tests/test_fp16.cpp:9-57 on the oracle
(oracle/p100_oracle.cpp) that every bit-exact parity test builds on."""
import math
import struct

import numpy as np
import pytest


def bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def from_bits(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


# (input, expected binary32 bits of the rounded value): overflow to inf at the
# 65520 tie, the subnormal/normal boundary, ties to even, underflow to zero.
PATTERNS = [
    (1.0, 0x3F800000), (65504.0, 0x477FE000), (65520.0, 0x7F800000), (-65520.0, 0xFF800000),
    (65519.0, 0x477FE000), (6.103515625e-5, 0x38800000), (6.1e-5, 0x387FC000), (5.96e-8, 0x33800000),
    (1.0 + 2.0 ** -11, 0x3F800000), (1.0 + 3.0 * 2.0 ** -11, 0x3F804000), (2.0 ** -25, 0x00000000),
    (-(2.0 ** -25), 0x80000000), (-0.0, 0x80000000), (from_bits(1), 0x00000000),
    (from_bits(0x7F7FFFFF), 0x7F800000), (-math.inf, 0xFF800000),
]


@pytest.mark.parametrize("x,expect", PATTERNS)
def test_known_patterns(orc, x, expect):
    assert bits(orc.fp16_round(x)) == expect


def test_nan_payload_kept(orc):
    nan = from_bits(0xFFC12345)
    assert bits(orc.fp16_round(nan)) == 0xFFC12345


def test_exhaustive_halves_and_ties(orc):
    # every finite half is a fixed point; midpoints round to even; neighbours
    # of a midpoint round to their side
    h = np.arange(0, 0x7BFF + 1, dtype=np.uint16).view(np.float16).astype(np.float32)
    r = orc.fp16_round
    for i in range(0, h.size, 7):   # a stride keeps the CPU suite fast; the ref test below covers the rest
        v = float(h[i])
        assert r(v) == v and bits(r(-v)) == bits(-np.float32(v))
        if i + 1 < h.size:
            nxt = float(h[i + 1])
            mid = float(np.float32((np.float32(v) + np.float32(nxt)) * np.float32(0.5)))
            even = v if i % 2 == 0 else nxt
            assert r(mid) == even and r(-mid) == -even
            assert r(float(np.nextafter(np.float32(mid), np.float32(v)))) == v
            assert r(float(np.nextafter(np.float32(mid), np.float32(nxt)))) == nxt


def test_half_bits_roundtrip(orc):
    for hb in list(range(0, 0x7C00, 97)) + [0x7C00, 0xFC00, 0x8001, 0x03FF, 0x0400]:
        v = orc.fp16_value(hb)
        assert orc.fp16_bits(v) == hb


def test_matches_reference_rounding(orc, ref):
    rng = np.random.default_rng(3)
    u32 = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32)
    f32 = u32.view(np.float32)
    specials = np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                         np.inf, -np.inf], np.float32)
    for x in np.concatenate([f32, specials, (rng.standard_normal(5000) * 1e3).astype(np.float32)]):
        x = float(x)
        a, b = orc.fp16_round(x), ref.round_to_fp16(x)
        assert bits(a) == bits(b) or (math.isnan(a) and math.isnan(b))
        assert orc.fp16_bits(x) == ref.half_bits(x) or math.isnan(x)
    for d in np.concatenate([rng.standard_normal(5000) * 10.0, rng.standard_normal(2000) * 1e-6,
                             [2.0 ** -25 + 2.0 ** -60, 65519.999999, -(2.0 ** -24) * 1.5]]):
        assert bits(orc.fp16_round_d(float(d))) == bits(ref.round_to_fp16_d(float(d)))
