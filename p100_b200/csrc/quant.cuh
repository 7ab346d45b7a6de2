// quant.cuh — Q8_1 activation quantisation and weight dequantisation.
//
// Both are bit-exact targets: the parity tests compare every output bit with
// the CPU contract (qmv_model.cpp:53-71 and :143).
#pragma once
#include "common.cuh"

namespace p100b {

// Q8_1 block of the 32 values a warp holds, one per lane (lane i = element
// i), written to the 36 bytes at blk.  Mirrors prepare() (qmv_model.cpp:53-71)
// and llama.cpp quantize.cu:88-110:
//   amax = max|x|, d = amax/127 (IEEE division), q = round-half-away(x/d),
//   sum  = XOR-butterfly (16,8,4,2,1) FP32 sum of the original x,
//   block = {fp16(d), fp16(sum), int8 q[32]}.
// No fast-math anywhere in this library: x/d and amax/127 stay IEEE.
__device__ __forceinline__ void warp_q8_1_block(float v, int lane, uint8_t* blk) {
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.0f;
    const int q = amax == 0.0f ? 0 : static_cast<int>(roundf(v / d));
    const float sum = warp_sum(v);
    if (lane == 0) {
        const uint32_t ds = uint32_t(__half_as_ushort(__float2half_rn(d))) |
                            (uint32_t(__half_as_ushort(__float2half_rn(sum))) << 16);
        *reinterpret_cast<uint32_t*>(blk) = ds;
    }
    blk[4 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
}

// One warp per 32-value block; 8 blocks per 256-thread CTA; blockIdx.y = row.
__global__ void __launch_bounds__(256) q8_1_quantize_kernel(const float* __restrict__ x,
                                                            uint8_t* __restrict__ out, int k, int blocks) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();   // x may come from the previous kernel
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    if (b >= blocks) return;
    const size_t row = blockIdx.y;
    const float v = x[row * size_t(k) + size_t(b) * 32 + lane];
    warp_q8_1_block(v, lane, out + (row * blocks + b) * 36);
}

// Six-bit scale and min of Q4_K sub-block j from the 12 packed bytes
// (qmv_model.cpp:72-77, get_scale_min_k4).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ float load_half_bytes(const uint8_t* p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// The 32 values of slab j (a Q4_0/Q8_0 block, or one 32-value sub-block of
// a Q4_K/Q5_K/Q6_K super-block) of a weight row: Q4_0 d*(nib-8), Q8_0 d*q,
// Q4_K/Q5_K fma(d*sc, q, -(dmin*mn)), Q6_K (d*sc)*q.  Each is the exact value
// rounded once to FP32, as float(double(...)) is in the model: the products
// are exact in FP32 and the double difference is exact for any fp16 d/dmin,
// so a single fused rounding gives the same bits.
template <int TYPE>
__device__ __forceinline__ void dequant_slab(const uint8_t* __restrict__ row, int j, float (&vals)[32]) {
    if (TYPE == P100_Q4_0) {
        const uint8_t* blk = row + size_t(j) * 18;
        const float d = load_half_bytes(blk);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int byte = blk[2 + i];
            vals[i] = d * float((byte & 15) - 8);
            vals[i + 16] = d * float((byte >> 4) - 8);
        }
    } else if (TYPE == P100_Q8_0) {
        const uint8_t* blk = row + size_t(j) * 34;
        const float d = load_half_bytes(blk);
#pragma unroll
        for (int i = 0; i < 32; ++i) vals[i] = d * float(static_cast<int8_t>(blk[2 + i]));
    } else if (TYPE == P100_Q4_K) {
        const uint8_t* blk = row + size_t(j / 8) * 144;
        const int sub = j % 8;
        const float d = load_half_bytes(blk), dmin = load_half_bytes(blk + 2);
        int sc, mn;
        q4k_scale_min(blk + 4, sub, sc, mn);
        const float ds = d * float(sc), ms = dmin * float(mn);
        const uint8_t* qs = blk + 16 + (sub / 2) * 32;
        const int shift = (sub % 2) * 4;
#pragma unroll
        for (int i = 0; i < 32; ++i) vals[i] = fmaf(ds, float((qs[i] >> shift) & 15), -ms);
    } else if (TYPE == P100_Q5_K) {
        // Q4_K's nibble plus 16 * bit `sub` of qh[i]; d*sc*q (<= 22 bits) and
        // dmin*mn are exact in FP32, so one fused rounding again
        const uint8_t* blk = row + size_t(j / 8) * 176;
        const int sub = j % 8;
        const float d = load_half_bytes(blk), dmin = load_half_bytes(blk + 2);
        int sc, mn;
        q4k_scale_min(blk + 4, sub, sc, mn);
        const float ds = d * float(sc), ms = dmin * float(mn);
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = blk + 48 + (sub / 2) * 32;
        const int shift = (sub % 2) * 4;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            vals[i] = fmaf(ds, float(((qs[i] >> shift) & 15) | (((qh[i] >> sub) & 1) << 4)), -ms);
    } else {
        // Q6_K slab 4h + c: ql[64h + 32(c&1) + i] nibble (c >= 2: high), bits
        // 4-5 from qh[32h + i] >> 2c, minus 32, times d * scales[8h + 2c + i/16];
        // d * sc (18 bits) times q (6 bits) is exact in FP32
        const uint8_t* blk = row + size_t(j / 8) * 210;
        const int sub = j % 8, h = sub / 4, c = sub % 4;
        const float d = load_half_bytes(blk + 208);
        const uint8_t* ql = blk + 64 * h + 32 * (c & 1);
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + 2 * c);
        const float ds0 = d * float(sc[0]), ds1 = d * float(sc[1]);
        const int nshift = (c >> 1) * 4, hshift = 2 * c;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int q = (((ql[i] >> nshift) & 15) | (((qh[i] >> hshift) & 3) << 4)) - 32;
            vals[i] = (i < 16 ? ds0 : ds1) * float(q);
        }
    }
}

// One thread per 32-value slab.
template <int TYPE>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ w, float* __restrict__ out,
                                                         int rows, int k, size_t row_bytes) {
    const int slabs = k / 32;
    const long long id = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= static_cast<long long>(rows) * slabs) return;
    const int r = static_cast<int>(id / slabs), j = static_cast<int>(id % slabs);
    float vals[32];
    dequant_slab<TYPE>(w + r * row_bytes, j, vals);
    float4* dst = reinterpret_cast<float4*>(out + size_t(r) * k + size_t(j) * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
}

}  // namespace p100b
