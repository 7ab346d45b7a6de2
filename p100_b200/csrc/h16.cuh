// h16.cuh — the FP16-activation mat-vec path (qmv::h16_model, the
// reference's own proposal, qmv_model.cpp:53-71,92-133).
//
// Activations: per 32-block, scale = max|x|, h = fp16(x / scale) stored in
// the 0,2,1,3 lane order of each group of four (bits 0 and 1 of the index
// swapped), and sum = the XOR-butterfly FP32 sum of the rounded h.  On the
// device: h as [batch][k] halves, then {scale, sum} as [batch][k/32] float2.
//
// Mat-vec, per 32-block of a row: two FP16 accumulators (the two halves of a
// half2) run HFMA2 chains of CHAIN steps over the element pairs of the
// stored order, each product-and-add rounded once to fp16 as the model's
// round_to_fp16(double(q) * h + acc); each chain ends as float(lo) +
// float(hi), times ds = (d * sc) * scale, added to the row in FP32
// (Q4_K: minus (dmin * mn) * scale * sum), in block order, with no
// contraction.  The stored order is what makes this cheap: a 32-bit word of
// quant bytes 4g..4g+3 yields the half2 pairs (4g, 4g+2) and (4g+1, 4g+3)
// with one mask each (the 0x6400 exponent trick turns a byte or nibble u
// into the half 1024 + u, and one exact half2 subtraction removes the
// offset).
//
// Layout: a lane owns a fixed 128-element column range (four 32-blocks) of
// every row, so its activations (64 half2 + four {scale, sum}) stay in
// registers for the whole launch; a team of k/128 lanes covers a row, and
// each lane reads its 72 (Q4_0), 136 (Q8_0) or 80 (Q4_K: header + half the
// quants of a super-block) bytes of the row with 8- or 16-byte loads, the
// next row's loads issued before the current row's arithmetic.  Within a
// lane the blocks are added in order; the team's lane sums are combined by
// a butterfly (and, past a warp, in fixed warp order): deterministic, and
// with one lane per row (k = 128) the row equals the model bit for bit.
#pragma once
#include "common.cuh"

namespace p100b {
namespace h16 {

constexpr int kThreads = 256;   // 8 warps: up to 255 registers a thread (Q8_0 holds two rows of 136 bytes)
constexpr int kWarps = kThreads / 32;
constexpr int kLaneElems = 128;   // elements per lane: four 32-blocks

__host__ __device__ constexpr int perm4(int i) { return (i & ~3) | ((i & 1) << 1) | ((i & 2) >> 1); }

// ------------------------------------------------------------ activations
// One warp per 32-block: x -> h (stored order), {scale, sum}.
__global__ void __launch_bounds__(256) h16_prepare_kernel(const float* __restrict__ x, __half* __restrict__ h,
                                                          float2* __restrict__ ss, int k, int nblocks_total) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const int lane = threadIdx.x & 31;
    const int blk = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (blk >= nblocks_total) return;   // whole warps leave together
    const float v = x[size_t(blk) * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const __half hv = amax == 0.0f ? __float2half_rn(0.0f) : __float2half_rn(__fdiv_rn(v, amax));
    h[size_t(blk) * 32 + perm4(lane)] = hv;
    const float sum = warp_sum(__half2float(hv));
    if (lane == 0) ss[blk] = make_float2(amax, sum);
}

// ------------------------------------------------------------ mat-vec
struct Params {
    const uint8_t* w;
    const __half* h;        // [k] halves of the column (stored order)
    const float2* ss;       // [k/32] {scale, sum}
    float* y;
    int rows, k;
    int row_bytes;
    int team;               // lanes per row: k / 128
    int team_pad;           // lanes per row rounded to a power of two (<= 32) or whole warps
};

__device__ __forceinline__ __half2 bits_h2(uint32_t v) {
    union {
        uint32_t u;
        __half2 h;
    } c;
    c.u = v;
    return c.h;
}

// The block's value: the model's chains, in FP32 as the model adds them.
// wq[j] = half2 of the weight quants at the stored pair j (exact small ints).
template <int CHAIN>
__device__ __forceinline__ float block_value(const __half2 (&wq)[16], const uint32_t (&hw)[16], float ds, float out) {
#pragma unroll
    for (int start = 0; start < 16; start += CHAIN) {
        __half2 acc = __float2half2_rn(0.0f);
#pragma unroll
        for (int j = start; j < start + CHAIN; ++j) acc = __hfma2(wq[j], bits_h2(hw[j]), acc);
        const float part = __fadd_rn(__low2float(acc), __high2float(acc));
        out = __fadd_rn(out, __fmul_rn(part, ds));
    }
    return out;
}

// Quants of one 32-block as the 16 half2 pairs of the stored order.
// Q4_0: word g of the 16 nibble bytes (g < 4) holds the low nibbles of
// elements 4g..4g+3 and the high nibbles of elements 16+4g..16+4g+3.
__device__ __forceinline__ void q4_0_pairs(const uint32_t (&qw)[4], __half2 (&wq)[16]) {
    const __half2 off = bits_h2(0x64086408u);   // 1032: the 1024 of the trick and the Q4_0 offset 8
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        wq[2 * g] = __hsub2(bits_h2((qw[g] & 0x000f000fu) | 0x64006400u), off);
        wq[2 * g + 1] = __hsub2(bits_h2(((qw[g] >> 8) & 0x000f000fu) | 0x64006400u), off);
        wq[8 + 2 * g] = __hsub2(bits_h2(((qw[g] >> 4) & 0x000f000fu) | 0x64006400u), off);
        wq[8 + 2 * g + 1] = __hsub2(bits_h2(((qw[g] >> 12) & 0x000f000fu) | 0x64006400u), off);
    }
}
// Q8_0: word g holds the codes of elements 4g..4g+3 (signed bytes).
__device__ __forceinline__ void q8_0_pairs(const uint32_t (&qw)[8], __half2 (&wq)[16]) {
    const __half2 off = bits_h2(0x64806480u);   // 1152 = 1024 + 128
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const uint32_t u = qw[g] ^ 0x80808080u;   // q + 128 per byte
        wq[2 * g] = __hsub2(bits_h2((u & 0x00ff00ffu) | 0x64006400u), off);
        wq[2 * g + 1] = __hsub2(bits_h2(((u >> 8) & 0x00ff00ffu) | 0x64006400u), off);
    }
}
// Q4_K sub-block: word g of its 32-byte quant chunk, nibble plane sh (0, 4).
__device__ __forceinline__ void q4_k_pairs(const uint32_t (&qw)[8], int sh, __half2 (&wq)[16]) {
    const __half2 off = bits_h2(0x64006400u);   // 1024
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        wq[2 * g] = __hsub2(bits_h2(((qw[g] >> sh) & 0x000f000fu) | 0x64006400u), off);
        wq[2 * g + 1] = __hsub2(bits_h2(((qw[g] >> (sh + 8)) & 0x000f000fu) | 0x64006400u), off);
    }
}

// Six-bit scale and min of Q4_K sub-block j (get_scale_min_k4,
// qmv_model.cpp:72-77) from the 12 packed bytes in words s0..s2 (bytes
// 0-3, 4-7, 8-11), by shifts so the words stay in registers.
__device__ __forceinline__ void k4_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        mn = (s1 >> (8 * j)) & 63;
    } else {
        const int t = 8 * (j - 4);
        sc = ((s2 >> t) & 15) | (((s0 >> (t + 6)) & 3) << 4);
        mn = ((s2 >> (t + 4)) & 15) | (((s1 >> (t + 6)) & 3) << 4);
    }
}

// Bytes a lane reads per row: its four 32-blocks (Q4_0 72, Q8_0 136) or, for
// Q4_K, the super-block header (16) and its half of the quants (64).
template <int TYPE>
__host__ __device__ constexpr int lane_words() { return TYPE == P100_Q4_0 ? 18 : TYPE == P100_Q8_0 ? 34 : 20; }

template <int TYPE>
__device__ __forceinline__ void load_lane(const uint8_t* row, int tl, uint32_t (&r)[lane_words<TYPE>()]) {
    if constexpr (TYPE == P100_Q4_0 || TYPE == P100_Q8_0) {
        constexpr int n = lane_words<TYPE>() / 2;   // 8-byte loads
        const uint2* p = reinterpret_cast<const uint2*>(row + size_t(tl) * lane_words<TYPE>() * 4);
#pragma unroll
        for (int i = 0; i < n; ++i) {
            const uint2 v = __ldcs(p + i);
            r[2 * i] = v.x;
            r[2 * i + 1] = v.y;
        }
    } else {
        const uint8_t* sb = row + size_t(tl / 2) * 144;
        const uint4 hd = __ldcs(reinterpret_cast<const uint4*>(sb));
        r[0] = hd.x;
        r[1] = hd.y;
        r[2] = hd.z;
        r[3] = hd.w;
        const uint4* q = reinterpret_cast<const uint4*>(sb + 16 + (tl & 1) * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldcs(q + i);
            r[4 + 4 * i] = v.x;
            r[5 + 4 * i] = v.y;
            r[6 + 4 * i] = v.z;
            r[7 + 4 * i] = v.w;
        }
    }
}

// This lane's part of a row: its four blocks, in order.
template <int TYPE, int CHAIN>
__device__ __forceinline__ float lane_row(const uint32_t (&r)[lane_words<TYPE>()], int tl, const uint32_t (&hw)[4][16],
                                          const float2 (&xs)[4]) {
    float out = 0.0f;
    __half2 wq[16];
    if constexpr (TYPE == P100_Q4_0) {
        // block b: bytes 18b..18b+17 of the lane's 72: d, then 16 nibble bytes
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int o = 18 * b;   // byte offset (even)
            uint32_t qw[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int at = o + 2 + 4 * g;   // 2-byte aligned
                qw[g] = (at & 2) ? __byte_perm(r[at >> 2], r[(at >> 2) + 1], 0x5432) : r[at >> 2];
            }
            const uint32_t dw = r[o >> 2];
            const float d = (o & 2) ? half_hi(dw) : half_lo(dw);
            q4_0_pairs(qw, wq);
            out = block_value<CHAIN>(wq, hw[b], __fmul_rn(d, xs[b].x), out);
        }
    } else if constexpr (TYPE == P100_Q8_0) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int o = 34 * b;
            uint32_t qw[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const int at = o + 2 + 4 * g;
                qw[g] = (at & 2) ? __byte_perm(r[at >> 2], r[(at >> 2) + 1], 0x5432) : r[at >> 2];
            }
            const uint32_t dw = r[o >> 2];
            const float d = (o & 2) ? half_hi(dw) : half_lo(dw);
            q8_0_pairs(qw, wq);
            out = block_value<CHAIN>(wq, hw[b], __fmul_rn(d, xs[b].x), out);
        }
    } else {
        const float d = half_lo(r[0]), dmin = half_hi(r[0]);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int j = (tl & 1) * 4 + b;   // sub-block of the super-block
            int sc, mn;
            k4_scale_min(r[1], r[2], r[3], j, sc, mn);
            uint32_t qw[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) qw[g] = r[4 + (b >> 1) * 8 + g];   // chunk j/2 of the lane's half
            q4_k_pairs(qw, (j & 1) * 4, wq);
            out = block_value<CHAIN>(wq, hw[b], __fmul_rn(__fmul_rn(d, float(sc)), xs[b].x), out);
            out = __fsub_rn(out, __fmul_rn(__fmul_rn(__fmul_rn(dmin, float(mn)), xs[b].x), xs[b].y));
        }
    }
    return out;
}

template <int TYPE, int CHAIN>
__global__ void __launch_bounds__(kThreads, 1) qmv_h16_kernel(const Params p) {
    extern __shared__ float s_part[];   // [kWarps] per-warp team partials
    pdl_allow_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int team_pad = p.team_pad;
    const int teams = kThreads / team_pad;
    const int team_id = tid / team_pad, tl = tid % team_pad;
    const bool live = tl < p.team;
    const int warps_per_team = team_pad > 32 ? team_pad / 32 : 1;

    // activations of this lane's four blocks (from the previous kernel)
    pdl_wait_prior_grid();
    uint32_t hw[4][16];
    float2 xs[4];
    const int blk0 = tl * 4;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        if (live) {
            const uint4* hp = reinterpret_cast<const uint4*>(p.h + size_t(blk0 + b) * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 v = hp[i];
                hw[b][4 * i] = v.x;
                hw[b][4 * i + 1] = v.y;
                hw[b][4 * i + 2] = v.z;
                hw[b][4 * i + 3] = v.w;
            }
            xs[b] = p.ss[blk0 + b];
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) hw[b][i] = 0u;
            xs[b] = make_float2(0.f, 0.f);
        }
    }

    // rows of this block, then of this team: r = r0 + team_id + teams * i
    const int r0 = static_cast<int>(static_cast<long long>(p.rows) * blockIdx.x / gridDim.x);
    const int r1 = static_cast<int>(static_cast<long long>(p.rows) * (blockIdx.x + 1) / gridDim.x);
    constexpr int NW = lane_words<TYPE>();
    uint32_t cur[NW], nxt[NW];
    int r = r0 + team_id;
    if (live && r < r1) load_lane<TYPE>(p.w + size_t(r) * p.row_bytes, tl, cur);
    // Every lane of a warp runs the same iterations (the warp's first team
    // has the most rows; a team past its last row computes nothing), so the
    // shuffles below always see the whole warp.
    const int lead = team_pad <= 32 ? (warp * 32) / team_pad : team_id;
    const int iters = max(0, (r1 - r0 - lead + teams - 1) / teams);
    for (int it = 0; it < iters; ++it, r += teams) {
        const int rn = r + teams;
        const bool row_ok = r < r1;
        if (live && rn < r1) load_lane<TYPE>(p.w + size_t(rn) * p.row_bytes, tl, nxt);
        float v = live && row_ok ? lane_row<TYPE, CHAIN>(cur, tl, hw, xs) : 0.0f;
        // the team's sum: butterfly inside the (padded) team or the warp
        const int width = team_pad < 32 ? team_pad : 32;
        for (int off = width / 2; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off, width));
        if (warps_per_team == 1) {
            if (tl == 0 && row_ok) p.y[r] = v;
        } else {
            if (lane == 0) s_part[warp] = v;
            // the team's warps meet at a named barrier of their own
            asm volatile("bar.sync %0, %1;" ::"r"(1 + team_id), "r"(team_pad) : "memory");
            if (tl == 0 && row_ok) {
                float t = s_part[warp];
                for (int w = 1; w < warps_per_team; ++w) t = __fadd_rn(t, s_part[warp + w]);
                p.y[r] = t;
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + team_id), "r"(team_pad) : "memory");
        }
#pragma unroll
        for (int i = 0; i < NW; ++i) cur[i] = nxt[i];
    }
}

}  // namespace h16
}  // namespace p100b
