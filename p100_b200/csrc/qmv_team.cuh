// qmv_team.cuh — batch-1 quantised mat-vec with register-resident activations.
//
// The decode mat-vec streams every weight byte once, so its instruction cost
// per byte of HBM is what matters:
//   * A lane owns one fixed 256-weight column group of every row (eight Q4_0 /
//     Q8_0 blocks or one Q4_K / Q5_K / Q6_K super-block), so its Q8_1 activations for that
//     group live in registers for the whole launch (loaded once, 16-byte
//     loads); no activation traffic in the inner loop.
//   * A team of T lanes (T = k/256 rounded up to a power of two, or to whole
//     warps past 32) covers one row; the eight consumer warps form 256/T
//     teams, and one stage of the ring holds one row per team (32-37 KB for
//     Q4_0/Q4_K, whole rows, contiguous).
//   * One producer warp streams stages HBM -> shared memory with untiled
//     bulk-async copies (L2 evict-first) into a ring of full/empty mbarrier
//     slots; every consumer warp visits every stage in order.  The producer
//     keeps at most kLookahead stages in flight beyond the newest landed one:
//     when every SM asks for its whole ring at once the memory system
//     interleaves all of it and the first stage lands late, so consumers
//     would start late; a short lookahead lets stage 0 land first.
//   * The activations come from the previous kernel (PDL).  Only the producer
//     waits for it, after it has issued the first kLookahead weight stages;
//     it then copies the Q8_1 row to shared memory with one bulk copy that
//     sits ahead of every later weight stage, so it is not queued behind the
//     stream (plain loads issued by the consumers at that point waited for
//     the SM's in-flight weight bytes: about 2 us instead of 0.5 us).
//   * The group count (k / 256) is a template parameter for the common
//     hidden sizes, which turns the team geometry and the activation
//     addressing into constants; 0 selects the runtime-shaped variant.
//   * A group is read with 128-bit shared loads at a 144- or 272-byte lane
//     stride (bank-conflict free; Q5_K 176 bytes); high nibbles are
//     multiplied in place by an unsigned x signed dp4a and the 16x factor
//     removed by one shift.  Q6_K groups (210 bytes) sit on the 2-byte grid
//     and are read as aligned 32-bit words re-aligned by a funnel shift
//     (group_dot_q6k).
//   * Batch > 1 of Q5_K / Q6_K (no tensor-core form) is one launch per
//     column (Params.col0) by the host.
//   * Rows are finished by an XOR butterfly inside the team (and, for teams of
//     several warps, a fixed-order add of the warps' partials), so the result
//     is deterministic.
// The arithmetic per 32-block is the q81 path of qmv::evaluate
// (qmv_model.cpp:147-180): exact int32 block dots, FP32 scaling.
//
// Fused RMSNorm (the decode step, k = 4096 or 8192): instead of reading a
// Q8_1 row, the consumers build it from the residual stream: v = x_in +
// delta, y = (v * 1/sqrt(sum v^2 / k + eps)) * w, quantised into shared
// memory; block 0 also writes v to x_out.  Every consumer warp stands in for
// four (eight) warps of rmsnorm_q8_1_kernel's 1024-thread layout, with its
// chunk order, warp butterfly, in-order sum of warp partials and octet
// quantiser, so the Q8_1 bytes equal that kernel's; the weight stream starts
// before the norm as usual.
#pragma once
#include "common.cuh"
#include "decode.cuh"

namespace p100b {
namespace qmvt {

constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxSlots = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kLookahead = 2;   // stages in flight past the newest landed one
// 32 warp partials of the fused norm, between the mbarriers (2 x 8 ring
// mbarriers + the activation one end at byte 136) and part_off (384).
constexpr int kNormScratchOff = 256;

// Lanes per row for a row of `ngroups` 256-weight groups: the next power of
// two up to a warp, whole warps beyond (the host plan uses the same rule).
__host__ __device__ constexpr int team_lanes(int ngroups) {
    return ngroups <= 32 ? (ngroups <= 1 ? 1 : 2 * team_lanes((ngroups + 1) / 2)) : (ngroups + 31) / 32 * 32;
}

// d = a (unsigned bytes) . b (signed bytes) + c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Q8_1 activations of one 256-value group (eight blocks).
struct GroupAct {
    int q[64];     // int8 codes, four per word, block-major
    float dx[8];   // fp16 block scale
    float m[8];    // Q4_0: -8 * fp16 block sum;  Q4_K, Q5_K: sum of the block's codes;  Q8_0: unused
    int s16[16];   // Q6_K: sums of the codes of each 16 values (its scales are per 16)
};

struct Params {
    const uint8_t* w;
    const uint8_t* xq;
    float* y;
    int rows, k;
    int col0;
    int row_bytes;
    int ngroups;        // k / 256
    int team;           // lanes per row
    int teams;          // rows per stage
    int nslot;
    int slot_bytes;
    int part_off, act_off, ring_off;   // act_off: the Q8_1 row in shared memory
    // Fused RMSNorm (norm_w not null; the Q8_1 row then comes from these):
    // x_in, delta (may be null), x_out (may be null; x_in != x_out), eps.
    const float* x_in;
    const float* delta;
    float* x_out;
    const float* norm_w;
    float eps;
    // Fused quantisation (x_f32 not null, norm_w null): the Q8_1 row is
    // built from these fp32 activations (16-byte aligned) instead of read.
    const float* x_f32;
    // Tensor-parallel push (the PUSH kernels, batch 1): the rows are a
    // partial sum of a row-parallel matrix; instead of y they go, tagged with
    // the exchange's epoch e, into slot [e & 1][rank] of every rank's peer
    // arena (the dec::PeerAr in device memory that ar points to; the reduce
    // runs in the next RMSNorm).
    const dec::PeerAr* ar;
};

// The Q8_1 row of p.x_f32 into xs by the 8 consumer warps: float4 chunk c
// (values 4c..4c+3, block c / 8) by lane c % 8 of an octet; octet_q8_1_block
// repeats q8_1_quantize_kernel's butterfly, so the bytes are that kernel's.
__device__ __forceinline__ void quantize_row(const Params& p, uint8_t* xs) {
    const int nc = p.k / 4;
    const float4* xr = reinterpret_cast<const float4*>(p.x_f32);
    for (int c0 = 0; c0 < nc; c0 += kConsumers * 32) {   // every consumer thread runs every pass
        const int c = c0 + static_cast<int>(threadIdx.x);
        const bool live = c < nc;
        const float4 x = live ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float v[4] = {x.x, x.y, x.z, x.w};
        dec::octet_q8_1_block(v, c & 7, live ? xs + size_t(c >> 3) * 36 : nullptr);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");   // the whole row is written
}

// The fused RMSNorm prologue: the Q8_1 row of rmsnorm(x_in + delta) * w into
// xs, by the 8 consumer warps (256 threads), bit-identical to
// rmsnorm_q8_1_kernel.  NG = k / 256 (16 or 32).
template <int NG>
__device__ __forceinline__ void fused_norm_row(const Params& p, uint8_t* xs, float* s_part) {
    constexpr int k = NG * 256;
    constexpr int kNC = k / 4;                    // float4 chunks
    constexpr int kPer = kNC / dec::kNormThreads; // chunks per thread of the 1024-thread layout
    constexpr int kVW = dec::kNormThreads / 32 / kConsumers;   // its warps per consumer warp
    static_assert(kNC % dec::kNormThreads == 0 && kPer <= dec::kNormChunks, "k");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4* xr = reinterpret_cast<const float4*>(p.x_in);
    const float4* dr = reinterpret_cast<const float4*>(p.delta);
    float4* xo = blockIdx.x == 0 ? reinterpret_cast<float4*>(p.x_out) : nullptr;
    float4 v[kVW][kPer];
#pragma unroll
    for (int j = 0; j < kVW; ++j) {
        const int vt = (warp + kConsumers * j) * 32 + lane;   // thread of the 1024-thread layout
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int c = vt + i * dec::kNormThreads;
            float4 x = xr[c];
            if (dr) {
                const float4 d4 = dr[c];
                x = make_float4(__fadd_rn(x.x, d4.x), __fadd_rn(x.y, d4.y), __fadd_rn(x.z, d4.z), __fadd_rn(x.w, d4.w));
            }
            if (xo) xo[c] = x;
            v[j][i] = x;
            s = fmaf(x.x, x.x, s);
            s = fmaf(x.y, x.y, s);
            s = fmaf(x.z, x.z, s);
            s = fmaf(x.w, x.w, s);
        }
        s = warp_sum(s);
        if (lane == 0) s_part[warp + kConsumers * j] = s;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
    float t = s_part[0];
    for (int i = 1; i < dec::kNormThreads / 32; ++i) t = __fadd_rn(t, s_part[i]);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, float(k)), p.eps)));
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll
    for (int j = 0; j < kVW; ++j) {
        const int vt = (warp + kConsumers * j) * 32 + lane;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int c = vt + i * dec::kNormThreads;
            const float4 wv = w4[c];
            const float y[4] = {__fmul_rn(__fmul_rn(v[j][i].x, r), wv.x), __fmul_rn(__fmul_rn(v[j][i].y, r), wv.y),
                                __fmul_rn(__fmul_rn(v[j][i].z, r), wv.z), __fmul_rn(__fmul_rn(v[j][i].w, r), wv.w)};
            dec::octet_q8_1_block(y, c & 7, xs + size_t(c >> 3) * 36);
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");   // the whole row is written
}

// Group g of a Q8_1 row held in shared memory.
template <int TYPE>
__device__ __forceinline__ void load_group_act(const uint8_t* xs, int g, GroupAct& a) {
    // Eight consecutive 36-byte blocks = 288 bytes = 18 aligned 16-byte loads.
    const uint4* src = reinterpret_cast<const uint4*>(xs + size_t(g) * 8 * 36);
    uint32_t u[72];
#pragma unroll
    for (int i = 0; i < 18; ++i) {
        const uint4 v = src[i];
        u[4 * i] = v.x;
        u[4 * i + 1] = v.y;
        u[4 * i + 2] = v.z;
        u[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        int sumq = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            a.q[8 * b + i] = static_cast<int>(u[9 * b + 1 + i]);
            sumq = __dp4a(a.q[8 * b + i], 0x01010101, sumq);
        }
        a.dx[b] = half_lo(u[9 * b]);
        a.m[b] = TYPE == P100_Q4_0                         ? -8.0f * half_hi(u[9 * b])
                 : TYPE == P100_Q4_K || TYPE == P100_Q5_K ? float(sumq)
                                                          : 0.f;
        if (TYPE == P100_Q6_K) {
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo = __dp4a(a.q[8 * b + i], 0x01010101, lo);
                hi = __dp4a(a.q[8 * b + 4 + i], 0x01010101, hi);
            }
            a.s16[2 * b] = lo;
            a.s16[2 * b + 1] = hi;
        }
    }
}

// Bytes of one 256-value group in a row: eight Q4_0 / Q8_0 blocks or one
// K-quant super-block.
template <int TYPE>
__host__ __device__ constexpr int group_bytes() {
    return TYPE == P100_Q4_0 ? 144 : TYPE == P100_Q8_0 ? 272 : TYPE == P100_Q4_K ? 144 : TYPE == P100_Q5_K ? 176 : 210;
}

// Q6_K super-block (ggml block_q6_K: ql[128], qh[64], int8 scales[16], fp16
// d) dotted with its group's activations.  A group starts 2-byte aligned
// only (210-byte stride), so it is read as 54 aligned words from the word
// boundary at or below it and re-aligned with a funnel shift; the last word
// read ends at most 6 bytes past the group (the ring keeps 16 bytes of slack
// after its last slot).  Value v of half n (v = 128n + 32c + l, c = 0..3,
// l = 0..31) has code (nibble c>>1 of ql[64n + 32(c&1) + l]) | (bits 2c..2c+1
// of qh[32n + l]) << 4, minus 32, and scale scales[v / 16]; per 32-value
// block b the integer sum sc_lo*(dot_lo - 32 s_lo) + sc_hi*(dot_hi - 32
// s_hi) is exact, then scaled by dx_b and finally by d.
__device__ __forceinline__ float group_dot_q6k(const uint8_t* __restrict__ grp, const GroupAct& a, float acc) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(grp);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;   // 0 or 16
    uint32_t w[53];
    uint32_t prev = base[0];
#pragma unroll
    for (int i = 0; i < 53; ++i) {
        const uint32_t next = base[i + 1];
        w[i] = __funnelshift_r(prev, next, sh);
        prev = next;
    }
    // words: ql 0..31, qh 32..47, scales 48..51, d = low half of word 52
    float sd = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int b = 4 * n + c;   // the 32-value block
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t ql = w[16 * n + 8 * (c & 1) + i], qh = w[32 + 8 * n + i];
                const uint32_t code = ((ql >> (4 * (c >> 1))) & 0x0f0f0f0fu) | (((qh >> (2 * c)) & 0x03030303u) << 4);
                if (i < 4) lo = __dp4a(static_cast<int>(code), a.q[8 * b + i], lo);
                else hi = __dp4a(static_cast<int>(code), a.q[8 * b + i], hi);
            }
            const uint32_t scw = w[48 + 2 * n + (c >> 1)];   // scales 8n + 2c, 8n + 2c + 1
            const int sc_lo = static_cast<int8_t>((scw >> (16 * (c & 1))) & 255);
            const int sc_hi = static_cast<int8_t>((scw >> (16 * (c & 1) + 8)) & 255);
            const int isum = sc_lo * (lo - 32 * a.s16[2 * b]) + sc_hi * (hi - 32 * a.s16[2 * b + 1]);
            sd = fmaf(a.dx[b], float(isum), sd);
        }
    }
    return fmaf(half_lo(w[52]), sd, acc);
}

// acc += (row's group at grp) . (the group's activations)
template <int TYPE>
__device__ __forceinline__ float group_dot(const uint8_t* __restrict__ grp, const GroupAct& a, float acc) {
    if constexpr (TYPE == P100_Q6_K) {
        return group_dot_q6k(grp, a, acc);
    } else {
    constexpr int kWords = group_bytes<TYPE>() / 4;
    uint32_t w[kWords];
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(grp + 16 * i);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
    }
    if (TYPE == P100_Q4_0) {
        // Pairs of 18-byte blocks at word 9p: A = (d lo(w[9p]), nibbles at +2),
        // B = (d hi(w[9p+4]), nibbles at words 9p+5..9p+8).
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const int base = 9 * pr, bA = 2 * pr, bB = 2 * pr + 1;
            int la = 0, ha = 0, lb = 0, hb = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // byte m: low nibble is element m, high nibble element m+16
                const uint32_t qa = shift2(w[base + i], w[base + i + 1]), qb = w[base + 5 + i];
                la = __dp4a(static_cast<int>(qa & 0x0f0f0f0fu), a.q[8 * bA + i], la);
                ha = dp4a_us(qa & 0xf0f0f0f0u, a.q[8 * bA + 4 + i], ha);
                lb = __dp4a(static_cast<int>(qb & 0x0f0f0f0fu), a.q[8 * bB + i], lb);
                hb = dp4a_us(qb & 0xf0f0f0f0u, a.q[8 * bB + 4 + i], hb);
            }
            // d_w * (d_x * sum(nib*q) - 8 * sum(x))
            acc = fmaf(half_lo(w[base]), fmaf(float(la + (ha >> 4)), a.dx[bA], a.m[bA]), acc);
            acc = fmaf(half_hi(w[base + 4]), fmaf(float(lb + (hb >> 4)), a.dx[bB], a.m[bB]), acc);
        }
    } else if (TYPE == P100_Q8_0) {
        // Pairs of 34-byte blocks at word 17p: A = (d lo(w[17p]), codes at +2),
        // B = (d hi(w[17p+8]), codes at words 17p+9..17p+16).
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const int base = 17 * pr, bA = 2 * pr, bB = 2 * pr + 1;
            int sa0 = 0, sa1 = 0, sb0 = 0, sb1 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                sa0 = __dp4a(static_cast<int>(shift2(w[base + i], w[base + i + 1])), a.q[8 * bA + i], sa0);
                sa1 = __dp4a(static_cast<int>(shift2(w[base + 4 + i], w[base + 5 + i])), a.q[8 * bA + 4 + i], sa1);
                sb0 = __dp4a(static_cast<int>(w[base + 9 + i]), a.q[8 * bB + i], sb0);
                sb1 = __dp4a(static_cast<int>(w[base + 13 + i]), a.q[8 * bB + 4 + i], sb1);
            }
            acc = fmaf(half_lo(w[base]) * a.dx[bA], float(sa0 + sa1), acc);
            acc = fmaf(half_hi(w[base + 8]) * a.dx[bB], float(sb0 + sb1), acc);
        }
    } else {
        // One super-block: w[0] = d | dmin, w[1..3] = twelve 6-bit scale/min
        // bytes, then (Q4_K) w[4 + 8q + i] = nibbles of sub-blocks 2q (low)
        // and 2q+1 (high); Q5_K puts qh[32] at words 4..11 (bit j of qh[l]
        // is the 16 of value l of sub-block j) and the nibbles at 12 + 8q + i.
        constexpr int kQs = TYPE == P100_Q5_K ? 12 : 4;
        float sd = 0.f, sm = 0.f;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            const int j0 = 2 * qq, j1 = 2 * qq + 1;
            // get_scale_min_k4 (qmv_model.cpp:72-77) for sub-blocks j0, j1
            int sc0, mn0, sc1, mn1;
            if (qq < 2) {
                sc0 = (w[1] >> (8 * j0)) & 63;
                mn0 = (w[2] >> (8 * j0)) & 63;
                sc1 = (w[1] >> (8 * j1)) & 63;
                mn1 = (w[2] >> (8 * j1)) & 63;
            } else {
                const int k0 = j0 - 4, k1 = j1 - 4;
                sc0 = ((w[3] >> (8 * k0)) & 15) | (((w[1] >> (8 * k0 + 6)) & 3) << 4);
                mn0 = ((w[3] >> (8 * k0 + 4)) & 15) | (((w[2] >> (8 * k0 + 6)) & 3) << 4);
                sc1 = ((w[3] >> (8 * k1)) & 15) | (((w[1] >> (8 * k1 + 6)) & 3) << 4);
                mn1 = ((w[3] >> (8 * k1 + 4)) & 15) | (((w[2] >> (8 * k1 + 6)) & 3) << 4);
            }
            int l0 = 0, l1 = 0, h0 = 0, h1 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t n0 = w[kQs + 8 * qq + i], n1 = w[kQs + 4 + 8 * qq + i];
                if constexpr (TYPE == P100_Q5_K) {
                    // five-bit codes: nibble | (bit j of qh[l]) << 4
                    const uint32_t b0 = w[4 + i], b1 = w[8 + i];
                    const uint32_t c00 = (n0 & 0x0f0f0f0fu) | (((b0 >> j0) & 0x01010101u) << 4);
                    const uint32_t c01 = (n1 & 0x0f0f0f0fu) | (((b1 >> j0) & 0x01010101u) << 4);
                    const uint32_t c10 = ((n0 >> 4) & 0x0f0f0f0fu) | (((b0 >> j1) & 0x01010101u) << 4);
                    const uint32_t c11 = ((n1 >> 4) & 0x0f0f0f0fu) | (((b1 >> j1) & 0x01010101u) << 4);
                    l0 = __dp4a(static_cast<int>(c00), a.q[8 * j0 + i], l0);
                    l1 = __dp4a(static_cast<int>(c01), a.q[8 * j0 + 4 + i], l1);
                    h0 = __dp4a(static_cast<int>(c10), a.q[8 * j1 + i], h0);
                    h1 = __dp4a(static_cast<int>(c11), a.q[8 * j1 + 4 + i], h1);
                } else {
                    l0 = __dp4a(static_cast<int>(n0 & 0x0f0f0f0fu), a.q[8 * j0 + i], l0);
                    l1 = __dp4a(static_cast<int>(n1 & 0x0f0f0f0fu), a.q[8 * j0 + 4 + i], l1);
                    h0 = dp4a_us(n0 & 0xf0f0f0f0u, a.q[8 * j1 + i], h0);
                    h1 = dp4a_us(n1 & 0xf0f0f0f0u, a.q[8 * j1 + 4 + i], h1);
                }
            }
            // sum_j dx_j * (dot_j * sc_j) and sum_j dx_j * (sumq_j * mn_j)
            // (qmv_model.cpp:175-178)
            sd = fmaf(a.dx[j0], float((l0 + l1) * sc0), sd);
            sd = fmaf(a.dx[j1], float(((h0 + h1) >> (TYPE == P100_Q5_K ? 0 : 4)) * sc1), sd);
            sm = fmaf(a.dx[j0], a.m[j0] * float(mn0), sm);
            sm = fmaf(a.dx[j1], a.m[j1] * float(mn1), sm);
        }
        acc = fmaf(half_lo(w[0]), sd, fmaf(-half_hi(w[0]), sm, acc));
    }
    return acc;
    }
}

// The bytes one stage copies: rows [first, first + nrows) widened to the
// 16-byte grid (bulk copies move whole 16-byte units).  Rows of Q4_0, Q8_0,
// Q4_K and Q5_K are whole units, so this is exactly those rows; Q6_K rows of
// k not a multiple of 2048 (tensor-parallel slices) start anywhere on the
// 2-byte grid, the stage then begins (first * row_bytes) % 16 bytes into its
// slot, and the host plan requires the matrix to end on the grid (so no copy
// reads past it).  src: the byte offset of the copy in w.
__device__ __forceinline__ uint32_t stage_span(const Params& p, int first, int nrows, size_t& src) {
    const size_t off = size_t(first) * p.row_bytes;
    src = off & ~size_t(15);
    return static_cast<uint32_t>(((off + size_t(nrows) * p.row_bytes + 15) & ~size_t(15)) - src);
}

// NG = k / 256 when compiled for one hidden size, 0 for any (runtime shape).
// PUSH: the tensor-parallel push epilogue (Params::ar) instead of y.
template <int TYPE, int NG, bool PUSH = false>
__global__ void __launch_bounds__(kThreads, 1) qmv_team_kernel(const Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    float* partial = reinterpret_cast<float*>(smem + p.part_off);   // [2][teams][warps per team]
    uint8_t* ring = smem + p.ring_off;
    constexpr int kGroupBytes = group_bytes<TYPE>();
    const int ngroups = NG > 0 ? NG : p.ngroups;
    const int team_size = NG > 0 ? team_lanes(NG) : p.team;
    const int teams = NG > 0 ? kConsumers * 32 / team_lanes(NG) : p.teams;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = static_cast<int>(static_cast<long long>(p.rows) * blockIdx.x / gridDim.x);
    const int r1 = static_cast<int>(static_cast<long long>(p.rows) * (blockIdx.x + 1) / gridDim.x);
    const int nst = (r1 - r0 + teams - 1) / teams;

    uint64_t* act_bar = full + 2 * kMaxSlots;
    if (tid == 0) {
        for (int s = 0; s < p.nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        mbar_init(act_bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_allow_dependents();

    if (warp == kConsumers) {
        // ---- producer
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            const int look = min(kLookahead, p.nslot - 1);
            // weights never depend on the previous kernel: the first stages go
            // out before waiting for it (free slots, nothing to wait for)
            const int pre = min(look, nst);
            for (int s = 0; s < pre; ++s) {
                const int first = r0 + s * teams;
                size_t src;
                const uint32_t bytes = stage_span(p, first, min(teams, r1 - first), src);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_load(ring + size_t(s) * p.slot_bytes, p.w + src, bytes, &full[s],
                          policy);
            }
            // the activations may come from the previous kernel (with the
            // fused norm or quantisation the consumers build them and the
            // barrier is unused)
            pdl_wait_prior_grid();
            const bool act_copy = !p.norm_w && !p.x_f32;
            if (act_copy) {
                asm volatile("fence.proxy.async.global;" ::: "memory");
                const uint32_t abytes = static_cast<uint32_t>(p.k / 32 * 36);
                mbar_arrive_expect_tx(act_bar, abytes);
                bulk_load(smem + p.act_off, p.xq + size_t(p.col0) * abytes, abytes, act_bar, policy);
            }
            int issued = pre;
            for (int s = pre; s < nst; ++s) {
                const int slot = s % p.nslot;
                // stage s - look has landed (its slot cannot have been refilled:
                // that needs stage s - look + nslot > s to be issued first)
                if (!mbar_wait(&full[(s - look) % p.nslot], ((s - look) / p.nslot) & 1)) break;
                if (s >= p.nslot && !mbar_wait(&empty[slot], ((s / p.nslot) - 1) & 1)) break;
                const int first = r0 + s * teams;
                size_t src;
                const uint32_t bytes = stage_span(p, first, min(teams, r1 - first), src);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load(ring + size_t(slot) * p.slot_bytes, p.w + src, bytes, &full[slot],
                          policy);
                issued = s + 1;
            }
            // no copy may still be writing shared memory when the block exits
            // (normally everything has landed: the consumers needed it)
            if (act_copy) mbar_wait(act_bar, 0);
            for (int s = max(0, issued - p.nslot); s < issued; ++s) mbar_wait(&full[s % p.nslot], (s / p.nslot) & 1);
        }
        return;
    }

    // ---- consumers: every write below follows the producer's wait for the
    // previous kernel through the activation barrier
    const int team = tid / team_size, tl = tid % team_size;
    const bool has_group = tl < ngroups;
    GroupAct act;
    if constexpr (NG == 16 || NG == 32) {
        if (p.norm_w) {
            // x_in and delta come from earlier kernels: every consumer waits
            pdl_wait_prior_grid();
            fused_norm_row<NG>(p, smem + p.act_off, reinterpret_cast<float*>(smem + kNormScratchOff));
        }
    }
    if (!p.norm_w && p.x_f32) {
        pdl_wait_prior_grid();   // x may come from an earlier kernel
        quantize_row(p, smem + p.act_off);
    }
    if (!p.norm_w && !p.x_f32) {
        const bool ok = mbar_wait(act_bar, 0);
        int any_timeout;
        if (team_size <= 32) {
            any_timeout = __any_sync(0xffffffffu, !ok);
        } else {
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.eq.u32 p, %1, 0;\n\t"
                "bar.red.or.pred q, 15, %2, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(any_timeout)
                : "r"(static_cast<unsigned>(ok)), "r"(kConsumers * 32)
                : "memory");
        }
        if (any_timeout) return;
    }
    // push: the epoch of this exchange (advanced by the previous RMSNorm,
    // complete once the previous kernel is)
    unsigned epoch = 0;
    if constexpr (PUSH) {
        pdl_wait_prior_grid();
        epoch = unsigned(*p.ar->epoch) + 1u;
    }
    auto put = [&](int row, float v) {
        if constexpr (PUSH) {
            const dec::PeerAr& ar = *p.ar;
            const unsigned long long w = dec::tag_word(epoch, v);
            for (int r = 0; r < ar.world; ++r)
                dec::st_word(ar.slots[r] + (size_t(epoch & 1u) * ar.world + ar.rank) * ar.n + row, w);
        } else {
            p.y[size_t(p.col0) * p.rows + row] = v;
        }
    };
    if (has_group) {
        load_group_act<TYPE>(smem + p.act_off, tl, act);
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) act.q[i] = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) act.dx[i] = act.m[i] = 0.f;
    }

    for (int s = 0; s < nst; ++s) {
        const int slot = s % p.nslot;
        const bool timed_out = !mbar_wait(&full[slot], (s / p.nslot) & 1);
        int any_timeout;
        if (team_size <= 32) {
            // a team lies inside one warp: the warp decides for itself
            any_timeout = __any_sync(0xffffffffu, timed_out);
        } else {
            // teams span warps that meet at a named barrier below: decide for
            // all consumer warps at once so no team is left there alone
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 p, %1, 0;\n\t"
                "bar.red.or.pred q, 15, %2, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(any_timeout)
                : "r"(static_cast<unsigned>(timed_out)), "r"(kConsumers * 32)
                : "memory");
        }
        if (any_timeout) break;
        const uint8_t* stage = ring + size_t(slot) * p.slot_bytes;
        const int first = r0 + s * teams;
        const int nr = min(teams, r1 - first);
        float acc = 0.f;
        if (team < nr && has_group)
            acc = group_dot<TYPE>(stage + ((size_t(first) * p.row_bytes) & 15) + size_t(team) * p.row_bytes +
                                      size_t(tl) * kGroupBytes, act, acc);
        // the stage's words are in registers: hand the slot back
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (team_size <= 32) {
            // teams are aligned lane ranges of one warp: butterfly inside them
            for (int off = team_size >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (tl == 0 && team < nr) put(first + team, acc);
        } else {
            const int wpt = team_size >> 5, wit = tl >> 5;
            float* part = partial + (size_t(s & 1) * teams + team) * wpt;
            const float v = warp_sum(acc);
            if (lane == 0) part[wit] = v;
            asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(team_size) : "memory");
            if (tl == 0 && team < nr) {
                float sum = 0.f;
                for (int i = 0; i < wpt; ++i) sum += part[i];
                put(first + team, sum);
            }
        }
    }
}

}  // namespace qmvt
}  // namespace p100b
