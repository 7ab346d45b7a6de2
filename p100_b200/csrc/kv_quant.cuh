// kv_quant.cuh — q8_0 / q4_0 K/V cache blocks: conversion to fp16 and the
// quantisation of new rows.
//
// Block formats (ggml): q8_0 = {fp16 d, int8 q[32]} (34 bytes), value q*d;
// q4_0 = {fp16 d, u8 qs[16]} (18 bytes), value i < 16 the low nibble of
// qs[i], value i >= 16 the high nibble of qs[i-16], minus 8, times d.  Blocks
// run along the head dimension, so a cache row of D values is D/32 blocks and
// its byte stride is D/32 * 34 (or 18): rows are only 2-byte aligned in
// general, which the loaders below respect.
#pragma once
#include "common.cuh"

namespace p100b {
namespace kvq {

template <int KV>
__host__ __device__ constexpr int block_bytes() {
    return KV == P100_KV_Q8_0 ? 34 : 18;
}

// Eight fp16 values from eight code bytes (x0 = bytes 0-3, x1 = 4-7; for
// q8_0 the int8 codes, for q4_0 one nibble per byte), each code * d rounded
// once to fp16.  A byte c placed under the exponent byte 0x64 is the half
// 1024 + c exactly; subtracting 1024 + 128 (q8_0, after flipping the sign
// bit: offset binary) or 1024 + 8 (q4_0) is exact and leaves the signed
// code, and one half multiply by d rounds the exact product to nearest even
// (no flush-to-zero form is used, so subnormal results are kept).  That is
// __float2half(float(code) * d) bit for bit, the FP32 product being exact
// (8-bit code times 11-bit significand) — dequant_nc.cu:32-48's arithmetic.
template <int KV>
__device__ __forceinline__ uint4 dequant8(uint32_t x0, uint32_t x1, uint32_t d2) {
    if (KV == P100_KV_Q8_0) {
        x0 ^= 0x80808080u;
        x1 ^= 0x80808080u;
    }
    uint32_t h[4] = {__byte_perm(x0, 0x64u, 0x4140), __byte_perm(x0, 0x64u, 0x4342),
                     __byte_perm(x1, 0x64u, 0x4140), __byte_perm(x1, 0x64u, 0x4342)};
    const uint32_t bias = KV == P100_KV_Q8_0 ? 0x64806480u : 0x64086408u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(h[i]) : "r"(bias));
        asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h[i]) : "r"(d2));
    }
    return make_uint4(h[0], h[1], h[2], h[3]);
}

// Which eight code bytes hold values 8c .. 8c+7 of a block (c = 0..3), as an
// offset from the block start, and the nibble shift (q4_0).
template <int KV>
__host__ __device__ constexpr int chunk_offset(int c) {
    return 2 + 8 * (KV == P100_KV_Q8_0 ? c : (c & 1));
}
template <int KV>
__host__ __device__ constexpr int chunk_shift(int c) {
    return KV == P100_KV_Q8_0 ? 0 : (c >> 1) * 4;
}
template <int KV>
__device__ __forceinline__ void isolate(uint32_t& x0, uint32_t& x1, int shift) {
    if (KV == P100_KV_Q4_0) {
        x0 = (x0 >> shift) & 0x0F0F0F0Fu;
        x1 = (x1 >> shift) & 0x0F0F0F0Fu;
    }
}

// ------------------------------------------------------------ conversion
// A view ne = [ne00 values, ne01 rows, ne02, ne03] of blocks with strides
// s01, s02, s03 (in blocks) -> contiguous fp16 (dequant_nc.cu:53-121).
struct ConvParams {
    const uint8_t* src;
    __half* dst;
    long long ne01, ne02, ne03, s01, s02, s03;
    int ne00, chunks;      // chunks = ne00 / 8 per row
    int units;             // ne01 * chunks per plane
};

// One thread per 8 consecutive outputs of kUnits rows-chunks (a CTA covers
// 256 * kUnits consecutive (row, chunk) units of a plane): all their loads —
// four 2-byte loads of the code bytes (blocks are only 2-byte aligned) and
// one of d each — are issued before any conversion, then one 16-byte store
// each; a warp's stores cover 512 contiguous bytes.  Grid (units / (256 *
// kUnits), planes).
constexpr int kUnits = 4;
template <int KV>
__global__ void __launch_bounds__(256) kv_to_f16_kernel(const ConvParams p) {
    constexpr int BB = block_bytes<KV>();
    const int u0 = blockIdx.x * 256 * kUnits + threadIdx.x;
    int i01[kUnits], ch[kUnits];
#pragma unroll
    for (int j = 0; j < kUnits; ++j) {
        const int u = min(u0 + j * 256, p.units - 1);
        i01[j] = u / p.chunks;
        ch[j] = u - i01[j] * p.chunks;
    }
    for (long long plane = blockIdx.y; plane < p.ne02 * p.ne03; plane += gridDim.y) {
        const long long i03 = plane / p.ne02, i02 = plane - i03 * p.ne02;
        const uint8_t* base = p.src + (i03 * p.s03 + i02 * p.s02) * BB;
        uint32_t x0[kUnits], x1[kUnits], d[kUnits];
#pragma unroll
        for (int j = 0; j < kUnits; ++j) {
            const uint8_t* blk = base + (i01[j] * p.s01 + (ch[j] >> 2)) * BB;
            const unsigned short* q = reinterpret_cast<const unsigned short*>(blk + chunk_offset<KV>(ch[j] & 3));
            x0[j] = uint32_t(__ldg(q)) | (uint32_t(__ldg(q + 1)) << 16);
            x1[j] = uint32_t(__ldg(q + 2)) | (uint32_t(__ldg(q + 3)) << 16);
            d[j] = __ldg(reinterpret_cast<const unsigned short*>(blk));
        }
#pragma unroll
        for (int j = 0; j < kUnits; ++j) {
            if (u0 + j * 256 >= p.units) break;
            isolate<KV>(x0[j], x1[j], chunk_shift<KV>(ch[j] & 3));
            const uint4 v = dequant8<KV>(x0[j], x1[j], d[j] | (d[j] << 16));
            *reinterpret_cast<uint4*>(p.dst + (plane * p.ne01 + i01[j]) * p.ne00 + ch[j] * 8) = v;
        }
    }
}

// ------------------------------------------------------------ quantisation
// One 32-value block per warp, lane j holding value j; writes the block at
// blk (2-byte aligned, as every block of a row of blocks is).  ggml's block quantisers as llama.cpp runs them for a
// quantised cache (cpy-utils.cuh quantize_f32_q8_0_block /
// quantize_f32_q4_0_block):
//   q8_0: d = max|x| / 127, q = roundf(x * (d ? 1/d : 0));
//   q4_0: d = v / -8 for the first v of largest |x|, q = min(15, trunc(x/d + 8.5)).
// IEEE division (the library is built without fast-math).
template <int KV>
__device__ __forceinline__ void quantize_block_warp(float x, int lane, uint8_t* blk) {
    float d;
    if (KV == P100_KV_Q8_0) {
        const float amax = warp_max(fabsf(x));
        d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        blk[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(roundf(x * id)));
    } else {
        float a = fabsf(x);
        int idx = lane;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, a, off);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
            if (oa > a || (oa == a && oi < idx)) {
                a = oa;
                idx = oi;
            }
        }
        const float at = __shfl_sync(0xffffffffu, x, idx);
        const float vmax = a > 0.0f ? at : 0.0f;   // never updated when every |x| is 0
        d = vmax / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const int q = min(15, static_cast<int>(static_cast<int8_t>(x * id + 8.5f)));
        const int hi = __shfl_down_sync(0xffffffffu, q, 16);
        if (lane < 16) blk[2 + lane] = static_cast<uint8_t>(q | (hi << 4));
    }
    if (lane == 0) store_half_bits(blk, d);
}

}  // namespace kvq
}  // namespace p100b
