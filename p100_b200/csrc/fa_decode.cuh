// fa_decode.cuh — split-K FlashAttention-vec decode over an fp16 GQA KV cache.
//
// Grid: (parts, batch * n_head_kv).  A CTA owns one contiguous key range of
// one kv head and serves every query head of that head's GQA group, so each
// K/V byte leaves HBM once.  K and V tiles of 64 keys stream HBM -> shared
// memory through untiled bulk-async copies into a ring of mbarrier stages.
//
// Per tile: logits in FP32 (8 threads per key, each owning D/8 dims of the
// query heads in registers, XOR-shuffle reduction), one warp per query head
// runs the online softmax (running max m, sum l, rescale alpha), then every
// thread accumulates P*V for a quad of dims over its share of the tile's keys
// in FP32.  This is the arithmetic of attention_tiled_model with FP32 QK,
// P and O (attention_tiled_model.cpp:145-179; p_fp16 = o_fp16_out =
// o_accum_fp16 = false).
//
// With more than one part, each CTA writes its unnormalised O, m and l to the
// workspace; the last CTA of a kv head (an atomic ticket, no waiting) merges
// the parts: global max M, weights exp(m_p - M), one division, LSE = M +
// log(den) (attention_tiled_model.cpp:183-222, fattn-common.cuh:963-977).
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "quant.cuh"

namespace p100b {
namespace fa {

constexpr int kThreads = 256;
constexpr int kTile = 64;

struct Params {
    const float* q;
    const __half* k;
    const __half* v;
    const float* mask;       // [seq_kv] row of the additive mask, or null
    float* o;
    float* lse;              // or null
    float* ws_o;             // [batch*nkv][parts][G][D]
    float* ws_ml;            // [batch*nkv][parts][G][2]
    unsigned* tickets;       // [batch*nkv], zero between calls
    int nkv, G, seq, parts, nstage;
    long long head_stride, batch_stride;   // elements
    float scale, softcap;
    // Decode chain: keys are [0, *len_dev + len_add) clamped to [0, seq], read
    // after the wait for the previous kernel (which may have appended the
    // newest row); the K/V stream then starts after that wait too.  Null:
    // seq keys, streamed before the wait.
    const int* len_dev;
    int len_add;
    // Fused decode step (fa_mma_kernel only; null otherwise): q points at the
    // raw fused QKV row [nq_total q heads | nkv k heads | nkv v heads] of
    // position pos = *len_dev; every CTA rotates its query heads by
    // rope_cs[pos] ((cos, sin) per adjacent pair, as rope_kv_append_kernel
    // does), the CTA of the last part rotates the kv head's k row and stores
    // it and the v row as fp16 into cache row pos before it reads K/V, and the
    // context is keys [0, pos].  o_q81, if set, receives o as Q8_1 blocks.
    const float2* rope_cs;
    int nq_total;
    uint8_t* o_q81;
    // fa_mma_kernel only: the parts of a kv head form one thread-block
    // cluster (gridDim.x == parts <= 16) and merge through distributed shared
    // memory instead of ws_o / ws_ml / tickets.
    int cluster_merge;
    // fa_mma_kernel over an fp16 cache: 4-d tensor maps (d, rows [0, seq),
    // kv heads, batch) of k and v, boxes of 64 values x one tile of rows,
    // 128-byte swizzle (set by the launcher).
    CUtensorMap tmk, tmv;
};

__device__ __forceinline__ void half8_to_float(const uint4 v, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Last CTA of kv head bk: merges the parts' partials {m, l, unnormalised O}
// into o (and lse) with the rebased combine of attention_tiled_model.cpp:
// 183-222: M = max m_p, den = sum_p exp(m_p - M) l_p, o = sum_p exp(m_p - M)
// O_p / den over parts in order (parts with l = 0 skipped).  All (m, l) are
// loaded at once and the weights kept in shared memory (scratch: at least
// 2 * parts * G + 2 * G + G * D floats), so the only loop over parts with global
// loads is the last, unrolled so its loads are in flight together.
template <int THREADS>
__device__ __forceinline__ void merge_parts(const Params& p, int bk, int G, int D, size_t row0, float* scratch) {
    const int tid = threadIdx.x;
    const int np = p.parts;
    const float* all_o = p.ws_o + size_t(bk) * np * G * D;
    const float* all_ml = p.ws_ml + size_t(bk) * np * G * 2;
    float* s_pm = scratch;            // [parts][G] m, then the weights
    float* s_pl = s_pm + np * G;      // [parts][G] l
    float* s_gm = s_pl + np * G;      // [G]
    float* s_den = s_gm + G;          // [G]
    for (int i = tid; i < np * G; i += THREADS) {
        s_pm[i] = __ldcg(all_ml + 2 * i);
        s_pl[i] = __ldcg(all_ml + 2 * i + 1);
    }
    __syncthreads();
    if (tid < G) {
        float gmax = -INFINITY;
        for (int q = 0; q < np; ++q) gmax = fmaxf(gmax, s_pm[q * G + tid]);
        float den = 0.f;
        for (int q = 0; q < np; ++q) {
            const float l = s_pl[q * G + tid];
            den += l == 0.f ? 0.f : expf(s_pm[q * G + tid] - gmax) * l;
        }
        s_gm[tid] = gmax;
        s_den[tid] = den;
        if (p.lse) p.lse[row0 + tid] = den == 0.f ? -INFINITY : gmax + logf(den);
    }
    __syncthreads();
    for (int i = tid; i < np * G; i += THREADS) {   // weights replace m
        const int h = i % G;
        s_pm[i] = s_pl[i] == 0.f ? 0.f : expf(s_pm[i] - s_gm[h]);
    }
    __syncthreads();
    float* s_out = s_den + G;         // [G][D] the merged o, for the Q8_1 epilogue
    for (int i = tid; i < G * D; i += THREADS) {
        const int h = i / D;
        float num = 0.f;
#pragma unroll 8
        for (int q = 0; q < np; ++q) {
            const float w = s_pm[q * G + h];
            const float v = __ldcg(all_o + size_t(q) * G * D + i);
            if (s_pl[q * G + h] != 0.f) num = fmaf(w, v, num);
        }
        const float den = s_den[h];
        const float o = den == 0.f ? 0.f : num / den;
        p.o[(row0 + h) * D + (i % D)] = o;
        s_out[i] = o;
    }
    if (tid == 0) p.tickets[bk] = 0;   // ready for the next call
    if (p.o_q81) {
        __syncthreads();
        for (int j = tid >> 5; j < G * D / 32; j += THREADS / 32)
            warp_q8_1_block(s_out[j * 32 + (tid & 31)], tid & 31, p.o_q81 + (row0 * D / 32 + j) * 36);
    }
}

template <int D, int GMAX>
__global__ void __launch_bounds__(kThreads, 1) fa_decode_kernel(const Params p) {
    constexpr int HPG0 = 512 / D;                         // heads whose query slices fit 64 registers
    constexpr int HPG = HPG0 < GMAX ? HPG0 : GMAX;        // heads per QK group
    constexpr int HG = (GMAX + HPG - 1) / HPG;            // QK head groups
    constexpr int CH = D / 64;                            // 8-dim chunks per slice thread
    constexpr int KP = 32 / HG;                           // keys per QK pass
    constexpr int QUADS = D / 4;
    constexpr int KGROUPS = kThreads / QUADS;
    constexpr int KPG = kTile / KGROUPS;                  // keys per PV group per tile
    constexpr int PST = 8;                                // P row stride (floats)
    static_assert(HG * KP == 32 && KGROUPS * KPG == kTile, "thread mapping");

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);                  // 4 barriers
    float* s_logit = reinterpret_cast<float*>(smem + 64);                 // [GMAX][kTile]
    float* s_p = s_logit + GMAX * kTile;                                  // [kTile][PST]
    float* s_alpha = s_p + kTile * PST;                                   // [8]
    float* s_m = s_alpha + 8;                                             // [8]
    float* s_l = s_m + 8;                                                 // [8]
    float* s_q = s_l + 8;                                                 // [GMAX][D]
    unsigned* s_flag = reinterpret_cast<unsigned*>(s_q + GMAX * D);
    const size_t head_bytes = ((64 + (GMAX * kTile + kTile * PST + 24 + GMAX * D + 4) * 4) + 127) & ~size_t(127);
    uint8_t* ring = smem + head_bytes;
    const size_t slot_bytes = size_t(2) * kTile * D * sizeof(__half);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bk = blockIdx.y, part = blockIdx.x;
    const int b = bk / p.nkv, kvh = bk % p.nkv;
    const int G = p.G;
    int seq = p.seq;
    if (p.len_dev) {
        pdl_wait_prior_grid();
        seq = min(max(*p.len_dev + p.len_add, 0), p.seq);
    }
    const int key0 = static_cast<int>(static_cast<long long>(seq) * part / p.parts);
    const int key1 = static_cast<int>(static_cast<long long>(seq) * (part + 1) / p.parts);
    const int ntiles = (key1 - key0 + kTile - 1) / kTile;
    const __half* kbase = p.k + b * p.batch_stride + kvh * p.head_stride;
    const __half* vbase = p.v + b * p.batch_stride + kvh * p.head_stride;

    if (tid == 0) {
        for (int s = 0; s < p.nstage; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    uint64_t policy = 0;
    auto issue = [&](int t) {
        const int slot = t % p.nstage;
        const int j0 = key0 + t * kTile;
        const int n = min(kTile, key1 - j0);
        const uint32_t bytes = static_cast<uint32_t>(n) * D * sizeof(__half);
        __half* dst = reinterpret_cast<__half*>(ring + slot * slot_bytes);
        mbar_arrive_expect_tx(&full[slot], 2 * bytes);
        bulk_load(dst, kbase + size_t(j0) * D, bytes, &full[slot], policy);
        bulk_load(dst + kTile * D, vbase + size_t(j0) * D, bytes, &full[slot], policy);
    };
    if (tid == 0) {
        policy = l2_evict_first_policy();
        for (int t = 0; t < min(p.nstage, ntiles); ++t) issue(t);
    }
    pdl_allow_dependents();
    pdl_wait_prior_grid();

    // Query heads of this group (zero for padding heads g >= G).
    const float* qg = p.q + (size_t(b) * p.nkv * G + size_t(kvh) * G) * D;
    for (int i = tid; i < GMAX * D; i += kThreads) s_q[i] = i < G * D ? qg[i] : 0.f;
    for (int i = tid; i < kTile * PST; i += kThreads) s_p[i] = 0.f;
    if (tid < 8) s_alpha[tid] = 1.f;
    __syncthreads();

    // QK mapping: slice s (D/8 dims), head group hg, key kk within a pass.
    const int sl = tid & 7, rest = tid >> 3;
    const int hg = rest / KP, kk = rest % KP;
    float qr[HPG][CH * 8];
#pragma unroll
    for (int i = 0; i < HPG; ++i)
#pragma unroll
        for (int c = 0; c < CH; ++c)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int h = hg * HPG + i;
                qr[i][c * 8 + e] = h < GMAX ? s_q[h * D + c * 64 + sl * 8 + e] : 0.f;
            }

    // PV mapping: a quad of dims and a group of keys.
    const int quad = tid % QUADS, kg = tid / QUADS;
    float acc[GMAX][4];
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[h][i] = 0.f;

    const float neg_inf = -INFINITY;
    float m_run = neg_inf, l_run = 0.f;   // meaningful in warp h < G for head h
    bool aborted = false;

    for (int t = 0; t < ntiles; ++t) {
        const int slot = t % p.nstage;
        const bool timed_out = !mbar_wait(&full[slot], (t / p.nstage) & 1);
        const __half* Ks = reinterpret_cast<const __half*>(ring + slot * slot_bytes);
        const __half* Vs = Ks + kTile * D;
        const int j0 = key0 + t * kTile;
        const int n = min(kTile, key1 - j0);

        // ---- logits
#pragma unroll
        for (int pass = 0; pass < kTile / KP; ++pass) {
            const int key = pass * KP + kk;
            float dot[HPG];
#pragma unroll
            for (int i = 0; i < HPG; ++i) dot[i] = 0.f;
            if (key < n) {
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    float kf[8];
                    half8_to_float(*reinterpret_cast<const uint4*>(Ks + key * D + c * 64 + sl * 8), kf);
#pragma unroll
                    for (int i = 0; i < HPG; ++i)
#pragma unroll
                        for (int e = 0; e < 8; ++e) dot[i] = fmaf(qr[i][c * 8 + e], kf[e], dot[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < HPG; ++i) {
                dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], 1);
                dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], 2);
                dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], 4);
            }
            float mine = dot[0];
#pragma unroll
            for (int i = 1; i < HPG; ++i)
                if (sl == i) mine = dot[i];
            const int h = hg * HPG + sl;
            if (sl < HPG && h < GMAX) {
                float x = neg_inf;
                if (key < n && h < G) {
                    x = mine * p.scale;
                    if (p.softcap > 0.f) x = p.softcap * tanhf(x / p.softcap);
                    if (p.mask) x += p.mask[j0 + key];
                }
                s_logit[h * kTile + key] = x;
            }
        }
        __syncthreads();

        // ---- online softmax, one warp per query head
        if (warp < G) {
            const float x0 = s_logit[warp * kTile + lane], x1 = s_logit[warp * kTile + lane + 32];
            const float tmax = warp_max(fmaxf(x0, x1));
            const float m_new = fmaxf(m_run, tmax);
            float alpha = 1.f, p0 = 0.f, p1 = 0.f;
            if (m_new != neg_inf) {   // no visible key yet: leave m, l, O untouched
                alpha = m_run == neg_inf ? 0.f : expf(m_run - m_new);
                p0 = expf(x0 - m_new);
                p1 = expf(x1 - m_new);
                l_run = l_run * alpha + warp_sum(p0 + p1);
                m_run = m_new;
            }
            s_p[lane * PST + warp] = p0;
            s_p[(lane + 32) * PST + warp] = p1;
            if (lane == 0) s_alpha[warp] = alpha;
        }
        __syncthreads();

        // ---- O = O * alpha + P V
#pragma unroll
        for (int h = 0; h < GMAX; ++h) {
            const float a = s_alpha[h];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[h][i] *= a;
        }
#pragma unroll
        for (int j = 0; j < KPG; ++j) {
            const int key = kg * KPG + j;
            if (key < n) {
                const uint2 raw = *reinterpret_cast<const uint2*>(Vs + key * D + quad * 4);
                const __half2* hv = reinterpret_cast<const __half2*>(&raw);
                const float2 v01 = __half22float2(hv[0]), v23 = __half22float2(hv[1]);
                float pr[8];
                const float4 pa = *reinterpret_cast<const float4*>(s_p + key * PST);
                pr[0] = pa.x; pr[1] = pa.y; pr[2] = pa.z; pr[3] = pa.w;
                if (GMAX > 4) {
                    const float4 pb = *reinterpret_cast<const float4*>(s_p + key * PST + 4);
                    pr[4] = pb.x; pr[5] = pb.y; pr[6] = pb.z; pr[7] = pb.w;
                }
#pragma unroll
                for (int h = 0; h < GMAX; ++h) {
                    acc[h][0] = fmaf(pr[h], v01.x, acc[h][0]);
                    acc[h][1] = fmaf(pr[h], v01.y, acc[h][1]);
                    acc[h][2] = fmaf(pr[h], v23.x, acc[h][2]);
                    acc[h][3] = fmaf(pr[h], v23.y, acc[h][3]);
                }
            }
        }
        if (__syncthreads_or(timed_out)) {   // uniform decision: every thread leaves together
            aborted = true;
            break;
        }
        if (tid == 0 && t + p.nstage < ntiles) issue(t + p.nstage);
    }
    if (aborted) {
        if (tid == 0)
            for (int s = 0; s < min(p.nstage, ntiles); ++s) (void)mbar_wait(&full[s], 0);
        return;
    }

    // ---- reduce the key groups' accumulators (ring is idle now)
    if (warp < G && lane == 0) {
        s_m[warp] = m_run;
        s_l[warp] = l_run;
    }
    float* red = reinterpret_cast<float*>(ring);   // [KGROUPS][GMAX][D]
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
        *reinterpret_cast<float4*>(red + (kg * GMAX + h) * D + quad * 4) =
            make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();

    const size_t row0 = size_t(b) * p.nkv * G + size_t(kvh) * G;   // first query head row
    if (p.parts == 1) {
        for (int i = tid; i < G * D; i += kThreads) {
            const int h = i / D, d = i % D;
            float sum = 0.f;
#pragma unroll
            for (int g = 0; g < KGROUPS; ++g) sum += red[(g * GMAX + h) * D + d];
            const float l = s_l[h];
            p.o[(row0 + h) * D + d] = l == 0.f ? 0.f : sum / l;
            if (d == 0 && p.lse) p.lse[row0 + h] = l == 0.f ? neg_inf : s_m[h] + logf(l);
        }
        return;
    }

    float* my_o = p.ws_o + (size_t(bk) * p.parts + part) * G * D;
    float* my_ml = p.ws_ml + (size_t(bk) * p.parts + part) * G * 2;
    for (int i = tid; i < G * D; i += kThreads) {
        const int h = i / D, d = i % D;
        float sum = 0.f;
#pragma unroll
        for (int g = 0; g < KGROUPS; ++g) sum += red[(g * GMAX + h) * D + d];
        my_o[i] = sum;
    }
    if (tid < G) {
        my_ml[2 * tid] = s_m[tid];
        my_ml[2 * tid + 1] = s_l[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned ticket = atomicAdd(&p.tickets[bk], 1u);
        s_flag[0] = ticket == static_cast<unsigned>(p.parts - 1);
    }
    __syncthreads();
    if (!s_flag[0]) return;
    __threadfence();

    // Last CTA of this kv head: merge the parts (the ring is idle).
    merge_parts<kThreads>(p, bk, G, D, row0, reinterpret_cast<float*>(ring));
}

}  // namespace fa
}  // namespace p100b
