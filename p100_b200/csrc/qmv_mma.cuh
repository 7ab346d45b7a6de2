// qmv_mma.cuh — batch 2..16 quantised mat-vec on the tensor cores:
// mma.sync m16n8k32 (int8 x int8 -> int32) with 16 weight rows as the M rows
// of A, 8 batch columns as the N columns of B (two column groups for batch
// 9..16), and one 32-element block (a Q4_0/Q8_0 block, a Q4_K sub-block) as
// K = 32.
//
// Why this form: a K = 32 step is exactly one scale block, so the int32
// result of a step is that block's integer dot for 16 rows x 8 columns, and
// the FP32 scaling of qmv::evaluate's q81 path (qmv_model.cpp:147-180) is
// applied per step in registers.  The A fragment a thread holds (elements
// 4t..4t+3 and 4t+16..4t+19 of rows g and g+8) is the low and the high
// nibbles of one 32-bit word of each row's Q4_0 block (the low nibbles of two
// words of a Q4_K chunk), so weights are unpacked in registers and touch
// shared memory once, as the bulk copies wrote them; the activation codes are
// the B fragments and stay in registers for the whole launch.  (tcgen05 takes
// its operands from shared memory or TMEM only, so 4-bit weights would have
// to be unpacked into shared memory first; with the per-block scale epilogue
// that round trip costs more than the weight stream at 16 columns.)
//
// Epilogue arithmetic per block and output pair (columns 2t, 2t+1 of a row):
// the int32 accumulators start at the bits of 1.5 * 2^23, so the mma leaves
// the float 1.5 * 2^23 + dot (exact for |dot| < 2^22); one packed f32x2 add
// recovers float(dot) for both columns, and packed f32x2 FMAs apply the
// activation scales and the row's weight scale.
//
// Layout: one producer warp copies the batch's Q8_1 rows (after the PDL
// wait) into the last ring slots, then streams stages of whole rows (16
// Q4_0/Q4_K or 8 Q8_0 rows) with one bulk copy per row into an mbarrier ring;
// rows land row_stride = bytes + 16 apart so that the rows an mma reads sit
// in distinct banks.  The consumers move the activations into registers and a
// per-block scale table, then release those slots to the ring.  Each
// consumer warp owns a contiguous share of the K blocks; per stage it
// accumulates the stage's rows x 16 columns, writes them to shared memory,
// and after a barrier the partials are added in warp order: deterministic.
//
// Long rows (k = 14336, 28672 at batch 16) do not fit one CTA's shared
// memory: the K range is then split over the CTAs of a thread-block cluster
// (one slice each, the same rows), and after the last stage each CTA sums
// its share of the rows over the slices through distributed shared memory,
// in slice order.
#pragma once
#include "common.cuh"

namespace p100b {
namespace qmvm {

constexpr int kMaxConsumers = 8;
constexpr int kMaxThreads = (kMaxConsumers + 1) * 32;
constexpr int kMaxSlots = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kLookahead = 2;          // stages in flight past the newest landed one
constexpr int kMaxBlocksPerWarp = 32;  // register-resident activation fragments
// Row pitch (floats) of the per-warp partials.
constexpr int kPartStride = 20;
constexpr uint32_t kBiasBits = 0x4B400000u;   // 1.5 * 2^23 as a float
constexpr float kBias = 12582912.0f;

// Weight rows per stage: one m16 tile of Q4_0/Q4_K rows (about 36 KB at
// k = 4096), 8 Q8_0 rows (the same bytes; the tile's upper half is zero).
__host__ __device__ constexpr int stage_rows(int type) { return type == P100_Q8_0 ? 8 : 16; }

// Bytes of `blocks` 32-element K blocks of one row.
__host__ __device__ constexpr int slice_bytes_of(int type, int blocks) {
    return type == P100_Q4_0 ? blocks * 18 : type == P100_Q8_0 ? blocks * 34 : blocks / 8 * 144;
}

// Threads a block may have: with 9 warps one SM sub-partition holds three of
// them, which caps a thread at 168 registers; 128 registers of activation
// fragments (BPW * column groups = 64) run with at most 7 consumer warps.
__host__ __device__ constexpr int max_threads(int bpw, int ncg) { return bpw * ncg >= 64 ? 256 : kMaxThreads; }

struct Params {
    const uint8_t* w;
    const uint8_t* xq;
    float* y;
    int rows, k, batch;
    int consumers;     // consumer warps; warp `consumers` is the producer
    int slices;        // K slices = CTAs per cluster (1: no split)
    int row_bytes;     // one row in global memory
    int slice_bytes;   // one row's K slice
    int row_stride;    // stage row pitch: slice_bytes + 16
    int act_stride;    // one column's Q8_1 slice + 16
    int nslot, slot_bytes, act_slot;   // the activations overlay slots [act_slot, nslot)
    int dm_off, part_off, res_off, scr_off, ring_off;
};

// ------------------------------------------------------------ packed f32x2
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t pk_bits(int lo, int hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float2 unpk(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// D = A(16x32: u8 nibbles or s8 codes) * B(32x8 s8 codes) + C, int32
template <bool A_U8>
__device__ __forceinline__ void mma_i8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    if (A_U8) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    }
}

// acc(row, columns c, c+1) += w * fma(dot, d8, m): the Q4_0 / Q8_0 step
// (qmv_model.cpp:151-161; m = -8 * fp16 sum for Q4_0, 0 for Q8_0).  `biased`
// holds 1.5 * 2^23 + dot for the two columns; dm = {d8(c), d8(c+1), m(c),
// m(c+1)}; w2 = {w, w}.
__device__ __forceinline__ void scale_step(uint64_t& acc, int biased0, int biased1, const float4& dm, uint64_t w2,
                                           uint64_t nbias) {
    uint64_t v = add2(pk_bits(biased0, biased1), nbias);
    v = fma2(v, pk(dm.x, dm.y), pk(dm.z, dm.w));
    acc = fma2(v, w2, acc);
}

// The Q4_K step (qmv_model.cpp:163-179): acc += (d*sc) * d8 * dot
// - (dmin*mn) * (d8 * sum of codes); dm = {d8(c), d8(c+1), s(c), s(c+1)},
// sc = {d*sc, d*sc, -dmin*mn, -dmin*mn} of the row.
__device__ __forceinline__ void scale_step_k(uint64_t& acc, int biased0, int biased1, const float4& dm,
                                             const float4& sc, uint64_t nbias) {
    uint64_t v = add2(pk_bits(biased0, biased1), nbias);
    v = mul2(v, pk(dm.x, dm.y));
    acc = fma2(v, pk(sc.x, sc.y), acc);
    acc = fma2(pk(dm.z, dm.w), pk(sc.z, sc.w), acc);
}

// Six-bit scale and min of Q4_K sub-block j (the get_scale_min_k4 rule of
// qmv_model.cpp:72-77) from the super-block header words h (d/dmin, then the
// 12 packed scale bytes), times d and dmin.
__device__ __forceinline__ void q4k_sub_scale(const uint4& h, int j, float& dsc, float& dmn) {
    int sc, mn;
    if (j < 4) {
        sc = (h.y >> (8 * j)) & 63;
        mn = (h.z >> (8 * j)) & 63;
    } else {
        const int s = 8 * (j - 4);
        sc = ((h.w >> s) & 15) | (((h.y >> (s + 6)) & 3) << 4);
        mn = ((h.w >> (s + 4)) & 15) | (((h.z >> (s + 6)) & 3) << 4);
    }
    dsc = half_lo(h.x) * float(sc);
    dmn = half_hi(h.x) * float(mn);
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float ld_cluster_f32(const float* local, int rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// BPW = 32-element K blocks per consumer warp: even; a multiple of 8 (whole
// super-blocks) for Q4_K.  NCG = column groups of 8 (1: batch <= 8).
template <int TYPE, int BPW, int NCG>
__global__ void __launch_bounds__(max_threads(BPW, NCG), 1) qmv_mma_kernel(const Params p) {
    static_assert(BPW % 2 == 0 && BPW <= kMaxBlocksPerWarp, "blocks per warp");
    static_assert(TYPE != P100_Q4_K || BPW % 8 == 0, "whole Q4_K super-blocks per warp");
    static_assert(NCG == 1 || NCG == 2, "column groups");
    constexpr int kBlk = TYPE == P100_Q4_0 ? 18 : 34;
    constexpr int kRows = stage_rows(TYPE);
    constexpr bool kHi = kRows == 16;        // rows g+8 of the m16 tile hold weights
    constexpr bool kNibbles = TYPE != P100_Q8_0;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    uint64_t* act_bar = empty + kMaxSlots;
    uint64_t* act_free = act_bar + 1;
    float4* dm = reinterpret_cast<float4*>(smem + p.dm_off);     // [slice blocks][8 column pairs]
    float* part = reinterpret_cast<float*>(smem + p.part_off);   // [2][consumers][kRows][kPartStride]
    float* res = reinterpret_cast<float*>(smem + p.res_off);     // [rows of this CTA][16]: K split only
    uint8_t* ring = smem + p.ring_off;
    uint8_t* act = ring + size_t(p.act_slot) * p.slot_bytes;     // [batch][act_stride]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nw = p.consumers, nct = nw * 32;
    const int nbs = nw * BPW;                                    // 32-blocks in this CTA's K slice
    const int slice = static_cast<int>(blockIdx.x) % p.slices;  // the cluster rank
    const int nrb = static_cast<int>(gridDim.x) / p.slices, rb = static_cast<int>(blockIdx.x) / p.slices;
    const int r0 = static_cast<int>(static_cast<long long>(p.rows) * rb / nrb);
    const int r1 = static_cast<int>(static_cast<long long>(p.rows) * (rb + 1) / nrb);
    const int nst = (r1 - r0 + kRows - 1) / kRows;

    if (tid == 0) {
        for (int s = 0; s < p.nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], nw);
        }
        mbar_init(act_bar, 1);
        mbar_init(act_free, nw);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_allow_dependents();

    if (warp == nw) {
        // ---- producer: the activations first (after the PDL wait: they may
        // come from the previous kernel), then the batch-1 team kernel's ring
        // and lookahead, one bulk copy per row (its lane).  A block of this
        // kernel fills an SM, so it never starts beside the previous grid and
        // weights issued before the wait would only delay the activations.
        const uint64_t policy = l2_evict_first_policy();
        const int look = min(kLookahead, p.nslot - 1);
        const uint8_t* wslice = p.w + size_t(slice) * p.slice_bytes;
        pdl_wait_prior_grid();
        if (lane == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(act_bar, static_cast<uint32_t>(p.batch * nbs * 36));
        }
        __syncwarp();
        if (lane < p.batch)
            bulk_load(act + size_t(lane) * p.act_stride, p.xq + (size_t(lane) * (p.k / 32) + size_t(slice) * nbs) * 36,
                      static_cast<uint32_t>(nbs * 36), act_bar, policy);
        auto issue = [&](int s) {
            const int slot = s % p.nslot;
            const int first = r0 + s * kRows;
            const int n = min(kRows, r1 - first);
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * p.slice_bytes));
            __syncwarp();
            if (lane < n)
                bulk_load(ring + size_t(slot) * p.slot_bytes + size_t(lane) * p.row_stride,
                          wslice + size_t(first + lane) * p.row_bytes, p.slice_bytes, &full[slot], policy);
        };
        const int pre = min(look, nst);
        for (int s = 0; s < pre; ++s) issue(s);
        int issued = pre;
        for (int s = pre; s < nst; ++s) {
            bool ok = mbar_wait(&full[(s - look) % p.nslot], ((s - look) / p.nslot) & 1);
            if (ok && s >= p.nslot) ok = mbar_wait(&empty[s % p.nslot], ((s / p.nslot) - 1) & 1);
            if (ok && s == p.act_slot) ok = mbar_wait(act_free, 0);   // first use of the activation slots
            if (__any_sync(0xffffffffu, !ok)) break;
            issue(s);
            issued = s + 1;
        }
        if (lane == 0) {   // no copy in flight when the block exits
            mbar_wait(act_bar, 0);
            for (int s = max(0, issued - p.nslot); s < issued; ++s) mbar_wait(&full[s % p.nslot], (s / p.nslot) & 1);
        }
        __syncwarp();
        if (p.slices == 1) return;
    } else {
        // ---- consumers.  A timeout is decided for all consumer warps at
        // once: they meet at barrier 1 every stage.
        auto any_of_consumers = [&](bool v) {
            int r;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 p, %1, 0;\n\t"
                "bar.red.or.pred q, 15, %2, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(r)
                : "r"(static_cast<unsigned>(v)), "r"(nct)
                : "memory");
            return r != 0;
        };
        const bool failed = any_of_consumers(!mbar_wait(act_bar, 0));
        const uint64_t nbias = pk(-kBias, -kBias);
        const int kb0 = warp * BPW;   // this warp's first block in the slice
        uint32_t bx[BPW][NCG][2];     // B fragments: codes of columns cg*8 + g
        if (!failed) {
            // {d8, d8, m, m} of column pair (2j, 2j+1) per block (columns >=
            // batch zero)
            for (int i = tid; i < nbs * 8; i += nct) {
                const int b = i >> 3, j = i & 7;
                float d8[2] = {0.f, 0.f}, m[2] = {0.f, 0.f};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = 2 * j + h;
                    if (c < p.batch) {
                        const uint32_t* blk =
                            reinterpret_cast<const uint32_t*>(act + size_t(c) * p.act_stride + b * 36);
                        d8[h] = half_lo(blk[0]);
                        if (TYPE == P100_Q4_0) m[h] = -8.0f * half_hi(blk[0]);
                        if (TYPE == P100_Q4_K) {
                            int sq = 0;
#pragma unroll
                            for (int q = 1; q <= 8; ++q) sq = __dp4a(static_cast<int>(blk[q]), 0x01010101, sq);
                            m[h] = d8[h] * float(sq);
                        }
                    }
                }
                dm[i] = make_float4(d8[0], d8[1], m[0], m[1]);
            }
#pragma unroll
            for (int j = 0; j < BPW; ++j) {
#pragma unroll
                for (int cg = 0; cg < NCG; ++cg) {
                    const int c = cg * 8 + g;
                    const uint32_t* cw =
                        reinterpret_cast<const uint32_t*>(act + size_t(c) * p.act_stride + (kb0 + j) * 36 + 4);
                    bx[j][cg][0] = c < p.batch ? cw[t] : 0u;
                    bx[j][cg][1] = c < p.batch ? cw[t + 4] : 0u;
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nct) : "memory");   // dm complete, activations read
        if (lane == 0) mbar_arrive(act_free);

        float4* scr = reinterpret_cast<float4*>(smem + p.scr_off) + warp * (16 * 8);   // Q4_K: [16 rows][8 sub]
        for (int s = 0; s < (failed ? 0 : nst); ++s) {
            const int slot = s % p.nslot;
            if (any_of_consumers(!mbar_wait(&full[slot], (s / p.nslot) & 1))) break;
            const uint8_t* stage = ring + size_t(slot) * p.slot_bytes;
            const uint8_t* row_lo = stage + size_t(g) * p.row_stride;       // row g of the m16 tile
            const uint8_t* row_hi = stage + size_t(g + 8) * p.row_stride;   // row g + 8 (Q4_0, Q4_K)
            uint64_t acc[2][NCG];   // rows g, g+8 x columns (cg*8 + 2t, +1)
#pragma unroll
            for (int cg = 0; cg < NCG; ++cg) acc[0][cg] = acc[1][cg] = 0ull;
            if constexpr (TYPE != P100_Q4_K) {
#pragma unroll
                for (int jp = 0; jp < BPW / 2; ++jp) {
                    const int b = kb0 + 2 * jp;   // even: the pair starts 4-byte aligned
                    const uint32_t* p0 = reinterpret_cast<const uint32_t*>(row_lo + size_t(b) * kBlk);
                    const uint32_t* p1 = reinterpret_cast<const uint32_t*>(row_hi + size_t(b) * kBlk);
                    // Weight scales of rows g (and g+8): block b in the low
                    // half of the pair's word 0, block b+1 in the high half of
                    // word 4 (Q4_0) or 8 (Q8_0).  Lane t = 0 of the row's quad
                    // loaded word 0 and lane t = 3 the other for the
                    // fragments; shuffles hand them to the quad, so shared
                    // memory serves only fragment words.
                    const int quad0 = lane & ~3, quad3 = lane | 3;
                    uint32_t aA[4], aB[4], sA0, sB0, sA1 = 0, sB1 = 0;
                    if (TYPE == P100_Q4_0) {
                        const uint32_t x0 = p0[t], x1 = p0[t + 1], x5 = p0[5 + t];
                        const uint32_t y0 = p1[t], y1 = p1[t + 1], y5 = p1[5 + t];
                        sA0 = __shfl_sync(0xffffffffu, x0, quad0);
                        sB0 = __shfl_sync(0xffffffffu, x1, quad3);   // word 4
                        sA1 = __shfl_sync(0xffffffffu, y0, quad0);
                        sB1 = __shfl_sync(0xffffffffu, y1, quad3);
                        const uint32_t nA0 = shift2(x0, x1), nA1 = shift2(y0, y1);
                        aA[0] = nA0 & 0x0f0f0f0fu;
                        aA[1] = nA1 & 0x0f0f0f0fu;
                        aA[2] = (nA0 >> 4) & 0x0f0f0f0fu;
                        aA[3] = (nA1 >> 4) & 0x0f0f0f0fu;
                        aB[0] = x5 & 0x0f0f0f0fu;
                        aB[1] = y5 & 0x0f0f0f0fu;
                        aB[2] = (x5 >> 4) & 0x0f0f0f0fu;
                        aB[3] = (y5 >> 4) & 0x0f0f0f0fu;
                    } else {
                        const uint32_t x0 = p0[t], x1 = p0[t + 1], x4 = p0[t + 4], x5 = p0[t + 5];
                        sA0 = __shfl_sync(0xffffffffu, x0, quad0);
                        sB0 = __shfl_sync(0xffffffffu, x5, quad3);   // word 8
                        aA[0] = shift2(x0, x1);
                        aA[2] = shift2(x4, x5);
                        aB[0] = p0[9 + t];
                        aB[2] = p0[13 + t];
                        aA[1] = aA[3] = aB[1] = aB[3] = 0u;
                    }
                    const float wA0 = half_lo(sA0), wB0 = half_hi(sB0);
                    const uint64_t wA0p = pk(wA0, wA0), wB0p = pk(wB0, wB0);
                    uint64_t wA1p = 0, wB1p = 0;
                    if (kHi) {
                        const float wA1 = half_lo(sA1), wB1 = half_hi(sB1);
                        wA1p = pk(wA1, wA1);
                        wB1p = pk(wB1, wB1);
                    }
#pragma unroll
                    for (int cg = 0; cg < NCG; ++cg) {
                        const float4 dmA = dm[b * 8 + cg * 4 + t], dmB = dm[(b + 1) * 8 + cg * 4 + t];
                        int dA[4] = {int(kBiasBits), int(kBiasBits), int(kBiasBits), int(kBiasBits)};
                        int dB[4] = {int(kBiasBits), int(kBiasBits), int(kBiasBits), int(kBiasBits)};
                        mma_i8<kNibbles>(dA, aA, bx[2 * jp][cg]);
                        mma_i8<kNibbles>(dB, aB, bx[2 * jp + 1][cg]);
                        // d: (row g, columns 2t, 2t+1), (row g+8, columns 2t, 2t+1)
                        scale_step(acc[0][cg], dA[0], dA[1], dmA, wA0p, nbias);
                        scale_step(acc[0][cg], dB[0], dB[1], dmB, wB0p, nbias);
                        if (kHi) {
                            scale_step(acc[1][cg], dA[2], dA[3], dmA, wA1p, nbias);
                            scale_step(acc[1][cg], dB[2], dB[3], dmB, wB1p, nbias);
                        }
                    }
                }
            } else {
#pragma unroll
                for (int sj = 0; sj < BPW / 8; ++sj) {
                    const int sb = warp * (BPW / 8) + sj;   // super-block within the slice
                    const uint32_t* p0 = reinterpret_cast<const uint32_t*>(row_lo + sb * 144);
                    const uint32_t* p1 = reinterpret_cast<const uint32_t*>(row_hi + sb * 144);
                    // lane (g, t) decodes sub-blocks 2t, 2t+1 of rows g and g+8
                    {
                        const uint4 h0 = *reinterpret_cast<const uint4*>(p0);
                        const uint4 h1 = *reinterpret_cast<const uint4*>(p1);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            float s0, m0, s1, m1;
                            q4k_sub_scale(h0, 2 * t + q, s0, m0);
                            q4k_sub_scale(h1, 2 * t + q, s1, m1);
                            scr[g * 8 + 2 * t + q] = make_float4(s0, s0, -m0, -m0);
                            scr[(g + 8) * 8 + 2 * t + q] = make_float4(s1, s1, -m1, -m1);
                        }
                    }
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int b = kb0 + sj * 8 + 2 * c;   // sub-blocks 2c (low nibbles) and 2c+1 (high)
                        const uint32_t lo0 = p0[4 + 8 * c + t], hi0 = p0[8 + 8 * c + t];
                        const uint32_t lo1 = p1[4 + 8 * c + t], hi1 = p1[8 + 8 * c + t];
                        const uint32_t aA[4] = {lo0 & 0x0f0f0f0fu, lo1 & 0x0f0f0f0fu, hi0 & 0x0f0f0f0fu,
                                                hi1 & 0x0f0f0f0fu};
                        const uint32_t aB[4] = {(lo0 >> 4) & 0x0f0f0f0fu, (lo1 >> 4) & 0x0f0f0f0fu,
                                                (hi0 >> 4) & 0x0f0f0f0fu, (hi1 >> 4) & 0x0f0f0f0fu};
                        const float4 sA0 = scr[g * 8 + 2 * c], sA1 = scr[(g + 8) * 8 + 2 * c];
                        const float4 sB0 = scr[g * 8 + 2 * c + 1], sB1 = scr[(g + 8) * 8 + 2 * c + 1];
#pragma unroll
                        for (int cg = 0; cg < NCG; ++cg) {
                            const float4 dmA = dm[b * 8 + cg * 4 + t], dmB = dm[(b + 1) * 8 + cg * 4 + t];
                            int dA[4] = {int(kBiasBits), int(kBiasBits), int(kBiasBits), int(kBiasBits)};
                            int dB[4] = {int(kBiasBits), int(kBiasBits), int(kBiasBits), int(kBiasBits)};
                            mma_i8<true>(dA, aA, bx[sj * 8 + 2 * c][cg]);
                            mma_i8<true>(dB, aB, bx[sj * 8 + 2 * c + 1][cg]);
                            scale_step_k(acc[0][cg], dA[0], dA[1], dmA, sA0, nbias);
                            scale_step_k(acc[1][cg], dA[2], dA[3], dmA, sA1, nbias);
                            scale_step_k(acc[0][cg], dB[0], dB[1], dmB, sB0, nbias);
                            scale_step_k(acc[1][cg], dB[2], dB[3], dmB, sB1, nbias);
                        }
                    }
                    __syncwarp();   // scr is rewritten for the next super-block
                }
            }
            // the stage's words are in registers: hand the slot back
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            // partials [row][col] of this warp, then the fixed-order sum
            float* pp = part + (size_t(s & 1) * nw + warp) * kRows * kPartStride;
#pragma unroll
            for (int cg = 0; cg < NCG; ++cg) {
                *reinterpret_cast<float2*>(pp + g * kPartStride + cg * 8 + 2 * t) = unpk(acc[0][cg]);
                if (kHi) *reinterpret_cast<float2*>(pp + (g + 8) * kPartStride + cg * 8 + 2 * t) = unpk(acc[1][cg]);
            }
            asm volatile("bar.sync 1, %0;" ::"r"(nct) : "memory");
            for (int o = tid; o < kRows * 16; o += nct) {
                const int row = o >> 4, col = o & 15;
                const int r = r0 + s * kRows + row;
                if (col < p.batch && r < r1) {
                    const float* pb = part + size_t(s & 1) * nw * kRows * kPartStride + row * kPartStride + col;
                    float sum = pb[0];
                    for (int w = 1; w < nw; ++w) sum += pb[w * kRows * kPartStride];
                    if (p.slices == 1)
                        p.y[size_t(col) * p.rows + r] = sum;
                    else
                        res[(r - r0) * 16 + col] = sum;
                }
            }
        }
    }
    if (p.slices > 1) {
        // K split: every thread of the cluster meets here after its last
        // stage; CTA `slice` then sums rows [n*slice/S, n*(slice+1)/S) of the
        // row block over the slices in slice order, and no CTA leaves while
        // another may still read its shared memory.
        cluster_sync_all();
        const int n = r1 - r0;
        const int q0 = n * slice / p.slices, q1 = n * (slice + 1) / p.slices;
        for (int o = tid; o < (q1 - q0) * 16; o += static_cast<int>(blockDim.x)) {
            const int row = q0 + (o >> 4), col = o & 15;
            if (col < p.batch) {
                float sum = ld_cluster_f32(res + row * 16 + col, 0);
                for (int q = 1; q < p.slices; ++q) sum += ld_cluster_f32(res + row * 16 + col, q);
                p.y[size_t(col) * p.rows + r0 + row] = sum;
            }
        }
        cluster_sync_all();
    }
}

}  // namespace qmvm
}  // namespace p100b
