// step.cuh — the whole batch-1 decode step as ONE persistent kernel per token.
//
// The graph-replayed decoder (decoder.cuh) runs about eight kernels per layer;
// each boundary costs a drain and a ramp of the 148 SMs (a kernel's CTAs
// cannot start before the previous kernel's CTAs leave their SM: both want
// most of its shared memory), which is about 3 us a kernel, ~25 us a layer,
// whatever the layer's bytes.  A tensor-parallel rank streams 1/N of the
// bytes but pays the same boundaries plus two cross-GPU exchanges a layer.
//
// Here one cooperative launch (one CTA per SM, every CTA resident) runs the
// step, and the phases meet at grid barriers instead of kernel boundaries:
//   per layer: RMSNorm -> QKV mat-vec | attention (RoPE, KV append, split-K
//   over CTAs, last-CTA merge, Q8_1) | O mat-vec | (all-reduce) RMSNorm ->
//   gate/up mat-vec | SwiGLU + Q8_1 | down mat-vec | (all-reduce)
//   then RMSNorm -> LM head -> argmax; the next token and position.
// Warp specialisation: one producer warp streams this CTA's whole weight
// schedule for the token — every matrix's row range and, per layer, its
// attention K/V tiles — through a ring of shared-memory slots with untiled
// bulk-async copies; weights do not depend on activations, so the stream
// never waits for a barrier, only for a free slot.  Eight consumer warps
// run the phases.  The HBM stream thus continues across phase boundaries.
//
// Arithmetic (bit-identical to the separate kernels where noted):
//   * RMSNorm + Q8_1: rmsnorm_q8_1_kernel's 1024-thread order (each consumer
//     warp stands in for four of its warps), so the Q8_1 rows are its bytes;
//   * mat-vecs: qmv_team_kernel's lane-per-256-group dot and team reduction
//     (qmv_model.cpp:147-180 per block), so every y equals p100_qmv's;
//   * SwiGLU + Q8_1: swiglu_q8_1_kernel's (own exp, warp quantiser);
//   * attention: FP32 SIMT (q rotated and scaled, scores, online softmax per
//     64-key tile, split-K parts merged by the rebased combine of
//     attention_tiled_model.cpp:183-222), within tolerance.h of
//     attention_reference; the new K/V row is rotated, rounded to fp16 and
//     used from shared memory, and stored into the cache for later tokens;
//   * argmax: lowest index among equal maxima, NaN never wins (argmax_kernel).
//
// Tensor parallelism (world > 1, one rank per GPU): the o and down mat-vecs
// are row-parallel (K split), so their outputs are partial sums.  Each
// consumer lane that finishes a row stores it into slot [e & 1][rank] of
// every rank's arena (NVLink peer stores, no multicast), the CTA fences at
// system scope and adds 1 to every rank's exchange counter; the next RMSNorm
// waits until its own counter has counted every CTA of every rank and adds
// the world slots in rank order (every rank holds the same bits).  The
// argmax candidates of the ranks meet the same way.  Counters are 64-bit and
// never reset: targets are cumulative, from bases kept in device memory.
//
// Every wait is bounded (1 s, %globaltimer).  A wait that runs out sets the
// device error flag and this decoder's abort word; every CTA then leaves at
// its next wait, the producer drains its copies, and later launches return
// at once (the decoder must be recreated).
#pragma once
#include "common.cuh"
#include "decode.cuh"
#include "qmv_team.cuh"
#include "quant.cuh"

namespace p100b {
namespace stp {

constexpr int kConsumers = 8;
constexpr int kCThreads = kConsumers * 32;   // 256 consumer threads
constexpr int kThreads = kCThreads + 32;     // + the producer warp
constexpr int kMaxSlots = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kTile = 64;                    // keys per attention tile
constexpr int kMaxRanks = 8;
constexpr int kMaxG = 8;                     // query heads per kv head
constexpr int kMaxD = 128;                   // head_dim
constexpr int kMaxParts = 256;               // attention parts per kv head
constexpr int kBarCons = 14;                 // named barrier of the 256 consumers
constexpr int kBarVote = 15;                 // named barrier of their votes
// shared memory: barriers at 0, small scratch at kMiscOff, then the
// activation / attention region, then the ring
constexpr int kMiscOff = 256;
constexpr int kActOff = 1024;

// One weight matrix of this rank in one format, with qmv_team_kernel's team
// geometry for its k (team lanes per row, rows per stage).
struct Mat {
    const uint8_t* w;
    int rows, k, row_bytes, ngroups, team, teams;
};

struct Layer {
    Mat qkv, o, gu, down;
    const float* attn_norm;
    const float* ffn_norm;
    __half* kc;   // this layer's K cache [nkv][max_ctx][hd]
    __half* vc;
};

struct Params {
    const Layer* layers;
    int n_layer;
    Mat lm;
    const float* out_norm;
    const uint8_t* embed;
    size_t embed_row_bytes;
    int embed_type;
    int hidden, nq, nkv, G, hd, ffn, vocab, vocab0, max_ctx;
    float eps, scale;
    const float2* rope;   // [max_ctx][hd / 2] (cos, sin)
    float* x0;            // residual stream between the two norms of a layer
    float* x1;            // residual stream after the first norm of a layer, and after the step
    float* delta;         // one rank: the o / down output
    float* qkv;
    uint8_t* attn_q81;
    float* gu;
    uint8_t* ffn_q81;
    float* logits;
    float* ws_o;          // attention partials [nkv][kMaxParts][G][hd]
    float* ws_ml;         // [nkv][kMaxParts][G][2]
    unsigned* tickets;    // [nkv], zero between uses
    float* cand;          // [grid][2] per-CTA argmax candidates
    int* pos;
    int* token;
    unsigned long long* bar;    // grid barrier counter
    unsigned long long* base;   // [0] bar and [1] own exchange counter at the start of the token
    int* abort_flag;
    int world, rank;
    float* slots[kMaxRanks];               // rank r: [2][world][hidden]
    float* cslots[kMaxRanks];              // rank r: [world][2]
    unsigned long long* xcount[kMaxRanks]; // rank r's exchange counter
    // shared memory plan
    int nslot, slot_bytes, ring_off;
};

// ------------------------------------------------------------ sync helpers
__device__ __forceinline__ void cons_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kBarCons), "n"(kCThreads) : "memory");
}
// OR of v over the 256 consumer threads, returned to all of them.
__device__ __forceinline__ bool cons_any(bool v) {
    unsigned r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<unsigned>(v)), "n"(kBarVote), "n"(kCThreads)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ bool aborted(const Params& p) {
    return *reinterpret_cast<volatile const int*>(p.abort_flag) != 0;
}
__device__ __forceinline__ void raise_abort(const Params& p) {
    atomicExch(&g_device_error, kDevErrTimeout);
    atomicExch(p.abort_flag, 1);
}

// Consumer thread 0 waits until *ctr >= target (bounded; the abort word ends
// it early), then every consumer learns the outcome.  Returns false on abort.
__device__ __noinline__ bool wait_counter(const Params& p, const unsigned long long* ctr, unsigned long long target,
                                          bool sys) {
    bool ok = true;
    if (threadIdx.x == 0) {
        if ((sys ? ld_acquire_sys(ctr) : ld_acquire_gpu(ctr)) < target) {
            const unsigned long long start = globaltimer_ns();
            for (int it = 0;; ++it) {
                if ((sys ? ld_acquire_sys(ctr) : ld_acquire_gpu(ctr)) >= target) break;
                if ((it & 15) == 15) {
                    if (aborted(p)) {
                        ok = false;
                        break;
                    }
                    if (globaltimer_ns() - start > kWaitLimitNs) {
                        raise_abort(p);
                        ok = false;
                        break;
                    }
                }
            }
        }
        if (ok) __threadfence();
    }
    return !cons_any(!ok);
}

// Grid barrier of the consumers of every CTA.  target: the counter value
// once every CTA has arrived (cumulative).
__device__ __forceinline__ bool grid_sync(const Params& p, unsigned long long& target) {
    target += gridDim.x;
    cons_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_gpu(p.bar, 1ull);
    }
    return wait_counter(p, p.bar, target, false);
}

// The all-reduce meeting point after a row-parallel mat-vec: one rank meets
// at a grid barrier; with several ranks every CTA of every rank arrives on
// every rank's counter (after a system-scope fence over its peer stores).
__device__ __forceinline__ bool exchange(const Params& p, unsigned long long& bar_t, unsigned long long& x_t) {
    if (p.world == 1) return grid_sync(p, bar_t);
    x_t += static_cast<unsigned long long>(p.world) * gridDim.x;
    __threadfence_system();   // this thread's peer stores, before the CTA's arrival
    cons_sync();
    if (threadIdx.x == 0)
        for (int r = 0; r < p.world; ++r) red_release_sys(p.xcount[r], 1ull);
    return wait_counter(p, p.xcount[p.rank], x_t, true);
}

// mbarrier phase wait for a consumer or the producer: bounded, abortable.
// The abort word (global memory) is read only once the wait has lasted
// kAbortPollNs: a poll on every round would delay each wake-up by an L2
// round trip.
constexpr unsigned long long kAbortPollNs = 20000;
__device__ __forceinline__ bool ring_wait(const Params& p, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        const unsigned long long waited = globaltimer_ns() - start;
        if (waited > kAbortPollNs) {
            if (aborted(p)) return false;
            if (waited > kWaitLimitNs) {
                raise_abort(p);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------ work split
// Rows [r0, r1) of a matrix for this CTA (the same split on both sides).
__device__ __forceinline__ void row_range(int rows, int& r0, int& r1) {
    r0 = static_cast<int>(static_cast<long long>(rows) * blockIdx.x / gridDim.x);
    r1 = static_cast<int>(static_cast<long long>(rows) * (blockIdx.x + 1) / gridDim.x);
}

// Attention work of this CTA over keys [0, L): kv head h, tiles [t0, t1) of
// kTile keys, part `part` of `parts`.  CTAs are dealt to heads in equal
// groups; a head's tiles are split over at most one part per two tiles.
struct AttnWork {
    int h, part, parts, t0, t1;
    bool active;
};
__device__ __forceinline__ AttnWork attn_work(const Params& p, int L) {
    AttnWork a;
    const int ntiles = (L + kTile - 1) / kTile;
    const int cph = max(1, static_cast<int>(gridDim.x) / p.nkv);
    a.parts = min(min(cph, kMaxParts), max(1, ntiles / 2));
    a.h = blockIdx.x / cph;
    a.part = blockIdx.x % cph;
    a.active = a.h < p.nkv && a.part < a.parts;
    a.t0 = a.active ? a.part * ntiles / a.parts : 0;
    a.t1 = a.active ? (a.part + 1) * ntiles / a.parts : 0;
    return a;
}


// ------------------------------------------------------------ producer
// Streams this CTA's schedule for the token through the ring, in the order
// the consumers use it.  One thread issues; slot s of stage n is reused for
// stage n + nslot once all eight consumer warps released it.
struct Ring {
    uint64_t* full;
    uint64_t* empty;
    uint8_t* base;
};

__device__ __noinline__ void producer(const Params& p, const Ring& ring, int L) {
    const uint64_t policy = l2_evict_first_policy();
    int stage = 0;
    bool ok = true;
    // one stage of `bytes` (+ `bytes2` at byte `off2` of the slot)
    auto issue = [&](const uint8_t* src, uint32_t bytes, const uint8_t* src2, uint32_t bytes2, uint32_t off2) {
        const int slot = stage % p.nslot;
        if (stage >= p.nslot && !ring_wait(p, &ring.empty[slot], ((stage / p.nslot) - 1) & 1)) {
            ok = false;
            return;
        }
        uint8_t* dst = ring.base + size_t(slot) * p.slot_bytes;
        mbar_arrive_expect_tx(&ring.full[slot], bytes + bytes2);
        bulk_load(dst, src, bytes, &ring.full[slot], policy);
        if (bytes2) bulk_load(dst + off2, src2, bytes2, &ring.full[slot], policy);
        ++stage;
    };
    auto matrix = [&](const Mat& m) {
        int r0, r1;
        row_range(m.rows, r0, r1);
        for (int first = r0; first < r1 && ok; first += m.teams) {
            const int nr = min(m.teams, r1 - first);
            issue(m.w + size_t(first) * m.row_bytes, static_cast<uint32_t>(nr) * m.row_bytes, nullptr, 0, 0);
        }
    };
    const AttnWork aw = attn_work(p, L);
    const uint32_t row_b = static_cast<uint32_t>(p.hd) * 2;
    for (int l = 0; l < p.n_layer && ok; ++l) {
        const Layer& ly = p.layers[l];
        matrix(ly.qkv);
        if (aw.active) {
            const size_t head = size_t(aw.h) * p.max_ctx * p.hd;
            for (int t = aw.t0; t < aw.t1 && ok; ++t) {
                const int n = min(kTile, L - t * kTile);
                const size_t at = head + size_t(t) * kTile * p.hd;
                issue(reinterpret_cast<const uint8_t*>(ly.kc + at), n * row_b, reinterpret_cast<const uint8_t*>(ly.vc + at),
                      n * row_b, kTile * row_b);
            }
        }
        if (ok) matrix(ly.o);
        if (ok) matrix(ly.gu);
        if (ok) matrix(ly.down);
    }
    if (ok) matrix(p.lm);
    // no copy may still be writing shared memory when the block exits
    for (int s = max(0, stage - p.nslot); s < stage; ++s) mbar_wait(&ring.full[s % p.nslot], (s / p.nslot) & 1);
}

// ------------------------------------------------------------ consumers
// The Q8_1 row of k values at q81 (global, written by other CTAs) into act.
__device__ __forceinline__ void load_act(const uint8_t* q81, int k, uint8_t* act) {
    const int n16 = k / 32 * 36 / 16;
    const uint4* src = reinterpret_cast<const uint4*>(q81);
    uint4* dst = reinterpret_cast<uint4*>(act);
    for (int i = threadIdx.x; i < n16; i += kCThreads) dst[i] = __ldcg(src + i);
    cons_sync();
}

// RMSNorm + Q8_1 of the hidden vector into act, in rmsnorm_q8_1_kernel's
// order: v = in (+ delta | + the world slots in rank order | the embedding
// row when layer 0), CTA 0 stores v to out; y = (v * r) * w, octets of lanes
// quantise 32-blocks.  Consumer warp cw stands in for warps cw + 8j of the
// 1024-thread layout; KC = float4 chunks per thread of that layout.  Every
// load of a pass is issued before its first use.
template <int TYPE_E>
__device__ __forceinline__ float4 embed_chunk(const Params& p, int tok, int c) {
    float vals[32];
    dequant_slab<TYPE_E>(p.embed + size_t(tok) * p.embed_row_bytes, c >> 3, vals);
    const int e = (c & 7) * 4;
    return make_float4(vals[e], vals[e + 1], vals[e + 2], vals[e + 3]);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

template <int KC>
__device__ __noinline__ void norm_row_t(const Params& p, const float* in, int embed_tok, const float* delta, int par,
                                        const float* w, float* out, uint8_t* act, float* s_part) {
    constexpr int kVT = dec::kNormThreads;          // virtual threads
    constexpr int kVW = kVT / 32 / kConsumers;      // virtual warps per consumer warp (4)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.hidden, nc = k / 4;
    float4 v[kVW][KC];
    auto chunk = [&](int j, int i) { return (warp + kConsumers * j) * 32 + lane + i * kVT; };
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    if (embed_tok >= 0) {
#pragma unroll
        for (int j = 0; j < kVW; ++j)
#pragma unroll
            for (int i = 0; i < KC; ++i) {
                const int c = chunk(j, i);
                float4 x = zero;
                if (c < nc) {
                    switch (p.embed_type) {
                        case P100_Q4_0: x = embed_chunk<P100_Q4_0>(p, embed_tok, c); break;
                        case P100_Q8_0: x = embed_chunk<P100_Q8_0>(p, embed_tok, c); break;
                        case P100_Q4_K: x = embed_chunk<P100_Q4_K>(p, embed_tok, c); break;
                        case P100_Q5_K: x = embed_chunk<P100_Q5_K>(p, embed_tok, c); break;
                        default: x = embed_chunk<P100_Q6_K>(p, embed_tok, c); break;
                    }
                }
                v[j][i] = x;
            }
    } else {
        const float4* x4 = reinterpret_cast<const float4*>(in);
#pragma unroll
        for (int j = 0; j < kVW; ++j)
#pragma unroll
            for (int i = 0; i < KC; ++i) {
                const int c = chunk(j, i);
                v[j][i] = c < nc ? __ldcg(x4 + c) : zero;
            }
        if (p.world == 1 && delta) {
            const float4* d4 = reinterpret_cast<const float4*>(delta);
            float4 d[kVW][KC];
#pragma unroll
            for (int j = 0; j < kVW; ++j)
#pragma unroll
                for (int i = 0; i < KC; ++i) {
                    const int c = chunk(j, i);
                    d[j][i] = c < nc ? __ldcg(d4 + c) : zero;
                }
#pragma unroll
            for (int j = 0; j < kVW; ++j)
#pragma unroll
                for (int i = 0; i < KC; ++i) v[j][i] = add4(v[j][i], d[j][i]);
        } else if (p.world > 1 && par >= 0) {
            // the world partial sums, added in rank order
            const float* sl = p.slots[p.rank] + size_t(par) * p.world * k;
            float4 d[kVW][KC];
#pragma unroll
            for (int j = 0; j < kVW; ++j)
#pragma unroll
                for (int i = 0; i < KC; ++i) {
                    const int c = chunk(j, i);
                    d[j][i] = c < nc ? __ldcg(reinterpret_cast<const float4*>(sl) + c) : zero;
                }
            for (int r = 1; r < p.world; ++r) {
                const float4* s4 = reinterpret_cast<const float4*>(sl + size_t(r) * k);
                float4 o[kVW][KC];
#pragma unroll
                for (int j = 0; j < kVW; ++j)
#pragma unroll
                    for (int i = 0; i < KC; ++i) {
                        const int c = chunk(j, i);
                        o[j][i] = c < nc ? __ldcg(s4 + c) : zero;
                    }
#pragma unroll
                for (int j = 0; j < kVW; ++j)
#pragma unroll
                    for (int i = 0; i < KC; ++i) d[j][i] = add4(d[j][i], o[j][i]);
            }
#pragma unroll
            for (int j = 0; j < kVW; ++j)
#pragma unroll
                for (int i = 0; i < KC; ++i) v[j][i] = add4(v[j][i], d[j][i]);
        }
    }
    // the norm weights, in flight during the reduction below
    float4 wv[kVW][KC];
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
    for (int j = 0; j < kVW; ++j)
#pragma unroll
        for (int i = 0; i < KC; ++i) {
            const int c = chunk(j, i);
            wv[j][i] = c < nc ? w4[c] : zero;
        }
    const bool writer = blockIdx.x == 0 && out;
#pragma unroll
    for (int j = 0; j < kVW; ++j) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < KC; ++i) {
            const int c = chunk(j, i);
            if (c < nc) {
                if (writer) reinterpret_cast<float4*>(out)[c] = v[j][i];
                s = fmaf(v[j][i].x, v[j][i].x, s);
                s = fmaf(v[j][i].y, v[j][i].y, s);
                s = fmaf(v[j][i].z, v[j][i].z, s);
                s = fmaf(v[j][i].w, v[j][i].w, s);
            }
        }
        s = warp_sum(s);
        if (lane == 0) s_part[warp + kConsumers * j] = s;
    }
    cons_sync();
    float t = s_part[0];
    for (int i = 1; i < kVT / 32; ++i) t = __fadd_rn(t, s_part[i]);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, float(k)), p.eps)));
#pragma unroll
    for (int j = 0; j < kVW; ++j) {
#pragma unroll
        for (int i = 0; i < KC; ++i) {
            if ((warp + kConsumers * j) * 32 + i * kVT >= nc) break;   // uniform over the warp
            const int c = chunk(j, i);
            const bool live = c < nc;
            const float y[4] = {__fmul_rn(__fmul_rn(v[j][i].x, r), wv[j][i].x),
                                __fmul_rn(__fmul_rn(v[j][i].y, r), wv[j][i].y),
                                __fmul_rn(__fmul_rn(v[j][i].z, r), wv[j][i].z),
                                __fmul_rn(__fmul_rn(v[j][i].w, r), wv[j][i].w)};
            dec::octet_q8_1_block(y, c & 7, live ? act + size_t(c >> 3) * 36 : nullptr);
        }
    }
    cons_sync();
}

__device__ __forceinline__ void norm_row(const Params& p, const float* in, int embed_tok, const float* delta, int par,
                                         const float* w, float* out, uint8_t* act, float* s_part) {
    const int kc = (p.hidden / 4 + dec::kNormThreads - 1) / dec::kNormThreads;
    switch (kc) {
        case 1: norm_row_t<1>(p, in, embed_tok, delta, par, w, out, act, s_part); break;
        case 2: norm_row_t<2>(p, in, embed_tok, delta, par, w, out, act, s_part); break;
        case 3: norm_row_t<3>(p, in, embed_tok, delta, par, w, out, act, s_part); break;
        default: norm_row_t<4>(p, in, embed_tok, delta, par, w, out, act, s_part); break;
    }
}

// One mat-vec phase over this CTA's rows of m, activations (Q8_1) in act:
// qmv_team_kernel's consumer loop.  mode 0: y[row] = sum; mode 1 (a
// row-parallel partial sum): one rank y[row], several ranks slot [par][rank]
// of every rank; mode 2 (LM head): y[row] and the running argmax (bv, bi).
template <int TYPE>
__device__ __noinline__ bool mv_phase(const Params& p, const Mat& m, const uint8_t* act, const Ring& ring, float* part,
                                      int& stage, float* y, int mode, int par, float& bv, int& bi) {
    const int tid = threadIdx.x, lane = tid & 31;
    constexpr int kGroupBytes = qmvt::group_bytes<TYPE>();
    const int team_size = m.team, teams = m.teams;
    const int team = tid / team_size, tl = tid % team_size;
    const bool has_group = tl < m.ngroups;
    qmvt::GroupAct a;
    if (has_group) {
        qmvt::load_group_act<TYPE>(act, tl, a);
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) a.q[i] = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) a.dx[i] = a.m[i] = 0.f;
    }
    int r0, r1;
    row_range(m.rows, r0, r1);
    bool failed = false;
    for (int first = r0; first < r1; first += teams) {
        const int slot = stage % p.nslot;
        const uint32_t parity = (stage / p.nslot) & 1;
        ++stage;
        const bool late = !ring_wait(p, &ring.full[slot], parity);
        // teams inside one warp decide per warp; teams of several warps meet
        // at named barriers below, so all consumers decide together
        const bool stop = team_size <= 32 ? __any_sync(0xffffffffu, late) != 0 : cons_any(late);
        if (stop) {
            failed = true;
            break;
        }
        const uint8_t* stg = ring.base + size_t(slot) * p.slot_bytes;
        const int nr = min(teams, r1 - first);
        float acc = 0.f;
        if (team < nr && has_group)
            acc = qmvt::group_dot<TYPE>(stg + size_t(team) * m.row_bytes + size_t(tl) * kGroupBytes, a, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring.empty[slot]);
        float sum = acc;
        if (team_size <= 32) {
            for (int off = team_size >> 1; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        } else {
            const int wpt = team_size >> 5, wit = tl >> 5;
            float* pp = part + (size_t(stage & 1) * teams + team) * wpt;
            const float v = warp_sum(acc);
            if (lane == 0) pp[wit] = v;
            asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(team_size) : "memory");
            if (tl == 0 && team < nr) {
                sum = 0.f;
                for (int i = 0; i < wpt; ++i) sum += pp[i];
            }
        }
        if (tl == 0 && team < nr) {
            const int row = first + team;
            if (mode == 1 && p.world > 1) {
                for (int r = 0; r < p.world; ++r)
                    p.slots[r][(size_t(par) * p.world + p.rank) * p.hidden + row] = sum;
            } else {
                y[row] = sum;
            }
            if (mode == 2 && dec::better(sum, row, bv, bi)) {
                bv = sum;
                bi = row;
            }
        }
    }
    return !cons_any(failed);
}

// SwiGLU + Q8_1 of this CTA's 32-blocks of the FFN slice (swiglu_q8_1_kernel's
// arithmetic), gate|up from p.gu into p.ffn_q81.
__device__ __noinline__ void swiglu_phase(const Params& p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.ffn / 32;
    const int b0 = static_cast<int>(static_cast<long long>(nb) * blockIdx.x / gridDim.x);
    const int b1 = static_cast<int>(static_cast<long long>(nb) * (blockIdx.x + 1) / gridDim.x);
    for (int b = b0 + warp; b < b1; b += kConsumers) {
        const int i = b * 32 + lane;
        const float g = __ldcg(p.gu + i), u = __ldcg(p.gu + p.ffn + i);
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, dec::dec_exp(-g)));
        warp_q8_1_block(__fmul_rn(silu, u), lane, p.ffn_q81 + size_t(b) * 36);
    }
}

// Attention shared-memory region (floats): q [kMaxG][kMaxD] (the merged
// output at the end) | scores, then probabilities, double-buffered
// [2][kMaxG][kTile] | m, l [kMaxG] | alpha [2][kMaxG] | new k and v rows
// (fp16, kMaxD each) | merge weights [kMaxParts][kMaxG].
constexpr int kAttnQ = 0;
constexpr int kAttnS = kAttnQ + kMaxG * kMaxD;
constexpr int kAttnM = kAttnS + 2 * kMaxG * kTile;
constexpr int kAttnL = kAttnM + kMaxG;
constexpr int kAttnA = kAttnL + kMaxG;
constexpr int kAttnKV = kAttnA + 2 * kMaxG;   // 16-byte aligned; kMaxD halves of k, then of v
constexpr int kAttnW = kAttnKV + kMaxD;       // the two fp16 rows take kMaxD floats
constexpr int kAttnFloats = kAttnW + kMaxParts * kMaxG;
static_assert(kAttnKV % 4 == 0, "16-byte aligned fp16 rows");

// Sum over the 32 lanes of each of NV values, scattered: five XOR stages that
// each halve the values a lane keeps (31 shuffles for NV = 32).  Afterwards
// a lane holds the full sums of indices lane * (NV / 32) + b (b < NV / 32)
// when NV >= 32, else of index lane / (32 / NV) in v[0].
template <int NV>
__device__ __forceinline__ void reduce_scatter(float (&v)[NV], int lane) {
#pragma unroll
    for (int st = 0; st < 5; ++st) {
        const int o = 16 >> st;
        constexpr int kDummy = 0;
        (void)kDummy;
        const int n = NV >> st;
        if (n >= 2) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
                if (i < n / 2) {
                    const float send = upper ? v[i] : v[i + n / 2];
                    const float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
}

// This CTA's part of the attention of kv head aw.h over keys [0, L), L =
// pos + 1; q, k, v of the step from p.qkv (rotated here), K/V tiles from the
// ring.  The new key (pos) comes from shared memory, and the CTA whose part
// holds it stores it into the cache.  One part: normalised and quantised
// here; several: partials to the workspace, and the CTA that takes the
// head's last ticket merges them and quantises the head's output.
//   scores: warp w takes keys w*8 .. w*8+7 of the tile; lane l the D/32
//     dimensions from l*D/32, with its slice of the G queries in registers;
//     the 8*G partial dots are finished by a reduce-scatter over the lanes;
//   softmax: warp g updates head g's running (m, l) over the tile;
//   P.V: thread (dp, hg) accumulates dimension pair dp of heads hg, hg + HS,
//     over the tile's keys with four independent chains.
template <int D, int G>
__device__ __noinline__ bool attn_phase(const Params& p, const Layer& ly, const AttnWork& aw, int pos, const Ring& ring,
                                        int& stage, float* region) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = pos + 1;
    float* s_q = region + kAttnQ;
    float* s_s = region + kAttnS;
    float* s_m = region + kAttnM;
    float* s_l = region + kAttnL;
    float* s_al = region + kAttnA;
    __half* s_kn = reinterpret_cast<__half*>(region + kAttnKV);
    __half* s_vn = s_kn + kMaxD;
    float* s_w = region + kAttnW;
    const float2* cs = p.rope + size_t(pos) * (D / 2);
    // q of the group's heads: rotated, then scaled (the fused attention
    // kernel's arithmetic); the new k rotated and, like v, rounded to fp16
    const float2* qg = reinterpret_cast<const float2*>(p.qkv + size_t(aw.h) * G * D);
    for (int i = tid; i < G * D / 2; i += kCThreads) {
        const float2 x = __ldcg(qg + i), t = cs[i % (D / 2)];
        s_q[2 * i] = __fsub_rn(__fmul_rn(x.x, t.x), __fmul_rn(x.y, t.y)) * p.scale;
        s_q[2 * i + 1] = __fadd_rn(__fmul_rn(x.x, t.y), __fmul_rn(x.y, t.x)) * p.scale;
    }
    const float2* kr = reinterpret_cast<const float2*>(p.qkv + (size_t(p.nq) + aw.h) * D);
    const float2* vr = reinterpret_cast<const float2*>(p.qkv + (size_t(p.nq) + p.nkv + aw.h) * D);
    for (int i = tid; i < D / 2; i += kCThreads) {
        const float2 x = __ldcg(kr + i), t = cs[i], v = __ldcg(vr + i);
        reinterpret_cast<__half2*>(s_kn)[i] =
            __halves2half2(__float2half_rn(__fsub_rn(__fmul_rn(x.x, t.x), __fmul_rn(x.y, t.y))),
                           __float2half_rn(__fadd_rn(__fmul_rn(x.x, t.y), __fmul_rn(x.y, t.x))));
        reinterpret_cast<__half2*>(s_vn)[i] = __halves2half2(__float2half_rn(v.x), __float2half_rn(v.y));
    }
    if (tid < G) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }
    cons_sync();
    const int ntiles = (L + kTile - 1) / kTile;
    if (aw.t1 == ntiles && tid < D / 2) {   // this part holds key pos: the cache row for later tokens
        const size_t at = (size_t(aw.h) * p.max_ctx + pos) * D;
        reinterpret_cast<__half2*>(ly.kc + at)[tid] = reinterpret_cast<const __half2*>(s_kn)[tid];
        reinterpret_cast<__half2*>(ly.vc + at)[tid] = reinterpret_cast<const __half2*>(s_vn)[tid];
    }
    constexpr int DPL = D / 32;    // dimensions per lane in the scores
    constexpr int NV = 8 * G;      // partial dots per lane: 8 keys x G heads
    float qr[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) qr[g][e] = s_q[g * D + lane * DPL + e];
    constexpr int DP = D / 2, HS = kCThreads / DP, NH = (G + HS - 1) / HS;
    const int dp = tid % DP, hg = tid / DP;
    float2 acc[NH];
#pragma unroll
    for (int i = 0; i < NH; ++i) acc[i] = make_float2(0.f, 0.f);
    bool failed = false;
    for (int t = aw.t0; t < aw.t1; ++t) {
        const int slot = stage % p.nslot;
        const uint32_t parity = (stage / p.nslot) & 1;
        ++stage;
        if (cons_any(!ring_wait(p, &ring.full[slot], parity))) {
            failed = true;
            break;
        }
        const int buf = t & 1;
        float* sb = s_s + buf * kMaxG * kTile;
        float* ab = s_al + buf * kMaxG;
        const __half* kt = reinterpret_cast<const __half*>(ring.base + size_t(slot) * p.slot_bytes);
        const __half* vt = kt + kTile * D;
        const int key0 = t * kTile, nk = min(kTile, L - key0);
        const bool has_new = key0 + nk == L;   // the tile's last key is pos
        // ---- scores
        float v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            const int j = warp * 8 + jj;
            if (j < nk) {
                const __half* krow = (has_new && j == nk - 1) ? s_kn : kt + j * D;
                float kf[DPL];
                if constexpr (DPL == 4) {
                    const uint2 u = *reinterpret_cast<const uint2*>(krow + lane * 4);
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                    kf[0] = a.x;
                    kf[1] = a.y;
                    kf[2] = b.x;
                    kf[3] = b.y;
                } else {
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(krow + lane * 2));
                    kf[0] = a.x;
                    kf[1] = a.y;
                }
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int e = 0; e < DPL; ++e) v[jj * G + g] = fmaf(qr[g][e], kf[e], v[jj * G + g]);
            }
        }
        reduce_scatter<NV>(v, lane);
        if constexpr (NV >= 32) {
#pragma unroll
            for (int b = 0; b < NV / 32; ++b) {
                const int idx = lane * (NV / 32) + b, j = warp * 8 + idx / G, g = idx % G;
                sb[g * kTile + j] = j < nk ? v[b] : -INFINITY;
            }
        } else if (lane % (32 / NV) == 0) {
            const int idx = lane / (32 / NV), j = warp * 8 + idx / G, g = idx % G;
            sb[g * kTile + j] = j < nk ? v[0] : -INFINITY;
        }
        cons_sync();
        // ---- online softmax of head `warp` over the tile
        if (warp < G) {
            float* row = sb + warp * kTile;
            const float a0 = row[lane], a1 = row[lane + 32];
            const float mo = s_m[warp], mn = fmaxf(mo, warp_max(fmaxf(a0, a1)));
            const float p0 = expf(a0 - mn), p1 = expf(a1 - mn);
            const float ls = warp_sum(p0 + p1);
            row[lane] = p0;
            row[lane + 32] = p1;
            if (lane == 0) {
                const float al = expf(mo - mn);
                ab[warp] = al;
                s_l[warp] = fmaf(s_l[warp], al, ls);
                s_m[warp] = mn;
            }
        }
        cons_sync();
        // ---- P.V
        const int nold = has_new ? nk - 1 : nk;
#pragma unroll
        for (int i = 0; i < NH; ++i) {
            const int g = hg + i * HS;
            if (g < G) {
                const float al = ab[g];
                const float* pr = sb + g * kTile;
                float2 c[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) c[u] = make_float2(0.f, 0.f);
                for (int j0 = 0; j0 < nold; j0 += 4) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if (j0 + u < nold) {
                            const float2 vv =
                                __half22float2(reinterpret_cast<const __half2*>(vt + (j0 + u) * D)[dp]);
                            const float pj = pr[j0 + u];
                            c[u].x = fmaf(pj, vv.x, c[u].x);
                            c[u].y = fmaf(pj, vv.y, c[u].y);
                        }
                    }
                }
                if (has_new) {
                    const float2 vv = __half22float2(reinterpret_cast<const __half2*>(s_vn)[dp]);
                    const float pj = pr[nk - 1];
                    c[0].x = fmaf(pj, vv.x, c[0].x);
                    c[0].y = fmaf(pj, vv.y, c[0].y);
                }
                acc[i].x = fmaf(acc[i].x, al, (c[0].x + c[1].x) + (c[2].x + c[3].x));
                acc[i].y = fmaf(acc[i].y, al, (c[0].y + c[1].y) + (c[2].y + c[3].y));
            }
        }
        // the slot's K and V are read; the other buffer serves the next tile
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring.empty[slot]);
    }
    if (cons_any(failed)) return false;
    const size_t hp = size_t(aw.h) * kMaxParts;
    if (aw.parts > 1) {
#pragma unroll
        for (int i = 0; i < NH; ++i) {
            const int g = hg + i * HS;
            if (g < G) reinterpret_cast<float2*>(p.ws_o + ((hp + aw.part) * G + g) * D)[dp] = acc[i];
        }
        if (tid < G) reinterpret_cast<float2*>(p.ws_ml)[(hp + aw.part) * G + tid] = make_float2(s_m[tid], s_l[tid]);
        __threadfence();
        cons_sync();
        int* s_last = reinterpret_cast<int*>(s_al);
        if (tid == 0) {
            const unsigned old = atomicAdd(&p.tickets[aw.h], 1u);
            *s_last = old == unsigned(aw.parts - 1);
            if (*s_last) __threadfence();
        }
        cons_sync();
        if (!*s_last) return true;
        // the last part merges: weights exp(m_p - M), denominator sum w_p l_p
        if (warp < G) {
            const float2* ml = reinterpret_cast<const float2*>(p.ws_ml);
            float mloc = -INFINITY;
            for (int q = lane; q < aw.parts; q += 32) mloc = fmaxf(mloc, __ldcg(ml + (hp + q) * G + warp).x);
            const float M = warp_max(mloc);
            float dl = 0.f;
            for (int q = lane; q < aw.parts; q += 32) {
                const float2 mv = __ldcg(ml + (hp + q) * G + warp);
                const float w = expf(mv.x - M);
                s_w[q * kMaxG + warp] = w;
                dl = fmaf(w, mv.y, dl);
            }
            const float den = warp_sum(dl);
            if (lane == 0) s_l[warp] = den;
        }
        cons_sync();
#pragma unroll
        for (int i = 0; i < NH; ++i) {
            const int g = hg + i * HS;
            if (g < G) {
                // parts in batches of 8 loads in flight (one L2 round trip a batch)
                float2 o = make_float2(0.f, 0.f);
                for (int q0 = 0; q0 < aw.parts; q0 += 8) {
                    float2 pv[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        pv[u] = q0 + u < aw.parts
                                    ? __ldcg(reinterpret_cast<const float2*>(p.ws_o + ((hp + q0 + u) * G + g) * D) + dp)
                                    : make_float2(0.f, 0.f);
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        if (q0 + u < aw.parts) {
                            const float w = s_w[(q0 + u) * kMaxG + g];
                            o.x = fmaf(w, pv[u].x, o.x);
                            o.y = fmaf(w, pv[u].y, o.y);
                        }
                    }
                }
                acc[i] = o;
            }
        }
        if (tid == 0) p.tickets[aw.h] = 0u;
    }
    // normalise into s_q (free now), quantise the group's heads (32-value
    // blocks, a warp each)
    float* s_out = s_q;
#pragma unroll
    for (int i = 0; i < NH; ++i) {
        const int g = hg + i * HS;
        if (g < G) {
            const float den = s_l[g];
            s_out[g * D + 2 * dp] = __fdiv_rn(acc[i].x, den);
            s_out[g * D + 2 * dp + 1] = __fdiv_rn(acc[i].y, den);
        }
    }
    cons_sync();
    for (int b = warp; b < G * D / 32; b += kConsumers)
        warp_q8_1_block(s_out[b * 32 + lane], lane, p.attn_q81 + (size_t(aw.h) * G * D / 32 + b) * 36);
    return true;
}

template <int D>
__device__ __forceinline__ bool attn_dispatch(const Params& p, const Layer& ly, const AttnWork& aw, int pos,
                                              const Ring& ring, int& stage, float* region) {
    switch (p.G) {
        case 1: return attn_phase<D, 1>(p, ly, aw, pos, ring, stage, region);
        case 2: return attn_phase<D, 2>(p, ly, aw, pos, ring, stage, region);
        case 4: return attn_phase<D, 4>(p, ly, aw, pos, ring, stage, region);
        default: return attn_phase<D, 8>(p, ly, aw, pos, ring, stage, region);
    }
}

// Waits (one thread, bounded, abortable) until *ctr >= target.
__device__ __forceinline__ bool wait_alone(const Params& p, const unsigned long long* ctr, unsigned long long target) {
    const unsigned long long start = globaltimer_ns();
    for (int it = 0; ld_acquire_sys(ctr) < target; ++it) {
        if ((it & 15) == 15 && (aborted(p) || globaltimer_ns() - start > kWaitLimitNs)) {
            if (!aborted(p)) raise_abort(p);
            return false;
        }
    }
    return true;
}

// One token.  Grid: one CTA per SM (cooperative launch); kThreads threads.
template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    float* part = reinterpret_cast<float*>(smem + kMiscOff);   // [2][8] multi-warp team partials
    float* s_part = part + 64;                                  // [32] norm partials
    float* s_bv = s_part + 32;                                  // [8] argmax per warp
    int* s_bi = reinterpret_cast<int*>(s_bv + 8);               // [8]
    int* s_state = s_bi + 8;                                    // [3] abort, pos, token
    uint8_t* act = smem + kActOff;
    const Ring ring{full, empty, smem + p.ring_off};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < p.nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        fence_barrier_init();
        s_state[0] = aborted(p);
        s_state[1] = *p.pos;
        s_state[2] = *p.token;
    }
    __syncthreads();
    if (s_state[0]) return;   // an earlier step of this decoder gave up
    const int pos = s_state[1], tok = s_state[2];
    if (pos < 0 || pos >= p.max_ctx || tok < 0 || tok >= p.vocab) {
        if (tid == 0 && blockIdx.x == 0) atomicExch(&g_device_error, kDevErrInput);
        return;
    }
    if (warp == kConsumers) {
        if (lane == 0) producer(p, ring, pos + 1);
        return;
    }
    unsigned long long bar_t = p.base[0], x_t = p.base[1];
    int stage = 0, ex = 0;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const AttnWork aw = attn_work(p, pos + 1);
    bool ok = true;
    for (int l = 0; l < p.n_layer && ok; ++l) {
        const Layer& ly = p.layers[l];
        if (l == 0) norm_row(p, nullptr, tok, nullptr, -1, ly.attn_norm, p.x1, act, s_part);
        else norm_row(p, p.x0, -1, p.delta, (ex - 1) & 1, ly.attn_norm, p.x1, act, s_part);
        ok = mv_phase<TYPE>(p, ly.qkv, act, ring, part, stage, p.qkv, 0, 0, bv, bi);
        if (ok) ok = grid_sync(p, bar_t);
        if (ok && aw.active) {
            ok = p.hd == 128 ? attn_dispatch<128>(p, ly, aw, pos, ring, stage, reinterpret_cast<float*>(act))
                             : attn_dispatch<64>(p, ly, aw, pos, ring, stage, reinterpret_cast<float*>(act));
        }
        if (ok) ok = grid_sync(p, bar_t);
        if (ok) {
            load_act(p.attn_q81, ly.o.k, act);
            ok = mv_phase<TYPE>(p, ly.o, act, ring, part, stage, p.delta, 1, ex & 1, bv, bi);
        }
        if (ok) ok = exchange(p, bar_t, x_t);
        ++ex;
        if (ok) {
            norm_row(p, p.x1, -1, p.delta, (ex - 1) & 1, ly.ffn_norm, p.x0, act, s_part);
            ok = mv_phase<TYPE>(p, ly.gu, act, ring, part, stage, p.gu, 0, 0, bv, bi);
        }
        if (ok) ok = grid_sync(p, bar_t);
        if (ok) {
            swiglu_phase(p);
            ok = grid_sync(p, bar_t);
        }
        if (ok) {
            load_act(p.ffn_q81, ly.down.k, act);
            ok = mv_phase<TYPE>(p, ly.down, act, ring, part, stage, p.delta, 1, ex & 1, bv, bi);
        }
        if (ok) ok = exchange(p, bar_t, x_t);
        ++ex;
    }
    if (ok) {
        norm_row(p, p.x0, -1, p.delta, (ex - 1) & 1, p.out_norm, p.x1, act, s_part);
        ok = mv_phase<TYPE>(p, p.lm, act, ring, part, stage, p.logits, 2, 0, bv, bi);
    }
    if (!ok) return;
    // this CTA's argmax candidate, then the grid's (CTA order), then the ranks'
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (dec::better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
    }
    cons_sync();
    if (tid == 0) {
        for (int w = 1; w < kConsumers; ++w)
            if (dec::better(s_bv[w], s_bi[w], bv, bi)) {
                bv = s_bv[w];
                bi = s_bi[w];
            }
        p.cand[2 * blockIdx.x] = bv;
        p.cand[2 * blockIdx.x + 1] = __int_as_float(bi);
    }
    if (!grid_sync(p, bar_t) || blockIdx.x != 0 || tid != 0) return;
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
        const float v = __ldcg(p.cand + 2 * c);
        const int i = __float_as_int(__ldcg(p.cand + 2 * c + 1));
        if (dec::better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    if (p.world > 1) {
        const int gi = bi == 0x7fffffff ? p.vocab0 : bi + p.vocab0;
        for (int r = 0; r < p.world; ++r) {
            p.cslots[r][2 * p.rank] = bv;
            p.cslots[r][2 * p.rank + 1] = __int_as_float(gi);
        }
        __threadfence_system();
        for (int r = 0; r < p.world; ++r) red_release_sys(p.xcount[r], 1ull);
        x_t += static_cast<unsigned long long>(p.world);
        if (!wait_alone(p, p.xcount[p.rank], x_t)) return;
        bv = -INFINITY;
        bi = 0x7fffffff;
        for (int r = 0; r < p.world; ++r) {
            const float v = __ldcg(p.cslots[p.rank] + 2 * r);
            const int i = __float_as_int(__ldcg(p.cslots[p.rank] + 2 * r + 1));
            if (dec::better(v, i, bv, bi)) {
                bv = v;
                bi = i;
            }
        }
    }
    *p.token = bi == 0x7fffffff ? 0 : bi;
    *p.pos = pos + 1;
    p.base[0] = bar_t;
    p.base[1] = x_t;
}

}  // namespace stp
}  // namespace p100b
