// kv_oracle.cpp — CPU restatement of the quantised K/V cache formats.
// TEST INFRASTRUCTURE ONLY: the parity tests call it as the checker of
// p100_b200/csrc/kv_quant.cuh and of FlashAttention over a quantised cache;
// nothing in the library calls it.
//
// Conversion to fp16 follows the reference's replay of llama.cpp's
// non-contiguous dequantisation (bench/micro/dequant_nc.cu):
// dequantize_q8_0 / dequantize_q4_0 (:32-48) give float(q) * d and
// (float(nib) - 8) * d, dequantize_block stores them with __float2half
// (:53-77), over the view geometry of :53-121 (block strides s01, s02, s03;
// output contiguous [i03][i02][i01][i00]).  Both products are exact in FP32
// (an 8-bit integer times an 11-bit significand), so each output is the
// exact product rounded once to binary16, nearest-even.
//
// Quantisation of new K/V rows is not in the reference (its cache is filled
// by llama.cpp); it restates ggml's published block quantisers as llama.cpp
// 79e2e74 runs them for a quantised cache (ggml-cuda cpy-utils.cuh
// quantize_f32_q8_0_block / quantize_f32_q4_0_block, the same arithmetic as
// ggml-quants.c quantize_row_q8_0_ref / quantize_row_q4_0_ref): parity of
// that step is unpinned.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "p100_oracle.h"

namespace {

int block_bytes(int t) { return t == P100O_KV_Q8_0 ? 34 : t == P100O_KV_Q4_0 ? 18 : 0; }

uint16_t get_u16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }
void put_u16(uint8_t* p, uint16_t v) {
    p[0] = uint8_t(v & 255);
    p[1] = uint8_t(v >> 8);
}

}  // namespace

extern "C" {

int p100o_kv_block_bytes(int kv_type) { return block_bytes(kv_type); }

int p100o_kv_to_f16(int kv_type, const void* src, int64_t ne00, int64_t ne01, int64_t ne02, int64_t ne03,
                    int64_t s01, int64_t s02, int64_t s03, uint16_t* dst) {
    const int bb = block_bytes(kv_type);
    if (!bb || ne00 <= 0 || ne00 % 32 || ne01 < 0 || ne02 < 0 || ne03 < 0) return -1;
    const uint8_t* base = static_cast<const uint8_t*>(src);
    for (int64_t i03 = 0; i03 < ne03; ++i03)
        for (int64_t i02 = 0; i02 < ne02; ++i02)
            for (int64_t i01 = 0; i01 < ne01; ++i01)
                for (int64_t ib = 0; ib < ne00 / 32; ++ib) {
                    const uint8_t* blk = base + (i03 * s03 + i02 * s02 + i01 * s01 + ib) * bb;
                    const float d = p100o_fp16_value(get_u16(blk));
                    uint16_t* y = dst + ((i03 * ne02 + i02) * ne01 + i01) * ne00 + ib * 32;
                    for (int i = 0; i < 32; ++i) {
                        float v;
                        if (kv_type == P100O_KV_Q8_0) {
                            v = float(int8_t(blk[2 + i])) * d;                  // dequant_nc.cu:35-38
                        } else {
                            const int vui = blk[2 + (i & 15)];                 // :43-47, value i and i+16
                            v = (float(i < 16 ? (vui & 15) : (vui >> 4)) - 8.0f) * d;
                        }
                        y[i] = p100o_fp16_bits(v);
                    }
                }
    return 0;
}

// The reference's block generator (dequant_nc.cu:144-149): one LCG state r,
// advanced before d = fp16(0.01 + (r >> 8) * 1e-9) and before every quant
// byte (the top 8 bits).  seed 12345 is the reference's.
void p100o_kv_lcg_blocks(int kv_type, size_t nblk, uint32_t seed, void* out) {
    const int bb = block_bytes(kv_type);
    uint8_t* p = static_cast<uint8_t*>(out);
    uint32_t r = seed;
    for (size_t b = 0; b < nblk; ++b, p += bb) {
        r = r * 1664525u + 1013904223u;
        put_u16(p, p100o_fp16_bits(0.01f + float(r >> 8) * 1e-9f));
        for (int i = 2; i < bb; ++i) {
            r = r * 1664525u + 1013904223u;
            p[i] = uint8_t(r >> 24);
        }
    }
}

// n values (n % 32 == 0) -> n / 32 blocks.
//   q8_0: amax = max|x|, d = amax / 127, id = d ? 1 / d : 0,
//         q = roundf(x * id) (half away from zero), stored d = fp16(d).
//   q4_0: vmax = the first x of largest |x|, d = vmax / -8, id as above,
//         q = min(15, trunc(x * id + 8.5)), byte j = q[j] | q[j + 16] << 4.
int p100o_kv_quantize(int kv_type, const float* x, size_t n, void* out) {
    const int bb = block_bytes(kv_type);
    if (!bb || n % 32) return -1;
    uint8_t* p = static_cast<uint8_t*>(out);
    for (size_t b = 0; b < n / 32; ++b, x += 32, p += bb) {
        if (kv_type == P100O_KV_Q8_0) {
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(x[j]));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            put_u16(p, p100o_fp16_bits(d));
            for (int j = 0; j < 32; ++j) p[2 + j] = uint8_t(int8_t(std::round(x[j] * id)));
        } else {
            float amax = 0.0f, vmax = 0.0f;
            for (int j = 0; j < 32; ++j)
                if (amax < std::fabs(x[j])) {
                    amax = std::fabs(x[j]);
                    vmax = x[j];
                }
            const float d = vmax / -8.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            put_u16(p, p100o_fp16_bits(d));
            for (int j = 0; j < 16; ++j) {
                const int q0 = std::min(15, int(int8_t(x[j] * id + 8.5f)));
                const int q1 = std::min(15, int(int8_t(x[j + 16] * id + 8.5f)));
                p[2 + j] = uint8_t(q0 | (q1 << 4));
            }
        }
    }
    return 0;
}

}  // extern "C"
