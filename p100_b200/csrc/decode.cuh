// decode.cuh — the glue of a batch-1 decode step around the mat-vecs and the
// attention kernel: residual add + RMSNorm + Q8_1, RoPE + KV-cache append,
// SwiGLU + Q8_1, argmax, embedding row, synthetic initialisation.
//
// The reference has no decode step (its contract stops at one mat-vec and
// one attention call), so these kernels follow Llama-3 as llama.cpp runs it
// and the CPU restatement in oracle/ mirrors them operation by operation:
//   * every floating-point step is written with explicit _rn intrinsics or
//     fmaf, so nothing is contracted differently from the restatement;
//   * reductions use a fixed order (thread-strided partial sums, XOR
//     butterfly, warps in order), which the restatement repeats;
//   * exp() inside SiLU is this file's own (Cody-Waite reduction + Taylor
//     polynomial), computed identically on both sides.
// With these rules RMSNorm+Q8_1, RoPE+append, SwiGLU+Q8_1 and argmax are
// bit-exact against the restatement.
//
// Every kernel is launched as a programmatic dependent (PDL) in the decode
// chain: it signals its dependents at once and reads nothing a previous
// kernel wrote before griddepcontrol.wait.  Since every kernel of the chain
// waits before it finishes, a kernel past its wait sees all earlier kernels
// complete, including the position counter and KV rows of earlier steps.
#pragma once
#include "common.cuh"
#include "quant.cuh"
#include "kv_quant.cuh"

namespace p100b {
namespace dec {

constexpr int kNormThreads = 1024;    // 32 warps; float4 chunk c belongs to thread c % 1024
constexpr int kArgmaxThreads = 1024;

// ------------------------------------------------- one-shot peer all-reduce
// Tensor-parallel sum of an n-float partial vector over `world` GPUs of one
// box through NVLink peer memory (CUDA IPC mappings).  Every rank owns an
// arena of tagged slots [2][world][n]: 64-bit words holding a value (low 32
// bits) and the epoch that wrote it (high 32 bits).  One 8-byte store is
// single-copy atomic, so a reader that sees the epoch it waits for also sees
// that store's value: no fence and no arrival counter between the push and
// the reduce (an earlier form fenced every pushing thread at system scope
// and counted arrivals; the fences cost about 14 us an exchange).
//   push (the row-parallel mat-vec's epilogue, qmv_team_kernel's PUSH
//     kernels, or ar_push_kernel after any other producer): value v of row i
//     goes to word [e&1][rank][i] of every rank as (e << 32) | bits(v);
//   reduce (rmsnorm_q8_1_kernel with ar.world > 0): polls, bounded, until
//     every word it needs carries epoch e, adds the world values in rank
//     order (the same order on every rank, so every rank holds the same
//     bits), then stores e as the completed epoch.
// e = completed epoch + 1 (so never 0, the tag of a zeroed arena), read from
// a device counter, so a replayed graph uses a new epoch every call.  Slots
// are double-buffered by e & 1: a rank writes epoch e+2 into a peer only
// after its own reduce of e+1, which saw every rank's push of e+1, which each
// rank made after its reduce of e had finished reading.
constexpr int kArMaxRanks = 8;
constexpr int kArBlocks = 8;
struct PeerAr {
    unsigned long long* slots[kArMaxRanks];   // rank r's tagged words [2][world][n]
    int world, rank, n;
    int* epoch;                 // this rank's completed-epoch counter
    unsigned long long wait_ns; // the reduce's wait limit (0: kWaitLimitNs)
};

__device__ __forceinline__ unsigned long long tag_word(unsigned e, float v) {
    return (static_cast<unsigned long long>(e) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_words2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Grid kArBlocks x 256; n % (4 * kArBlocks) == 0.
__global__ void __launch_bounds__(256) ar_push_kernel(const float* __restrict__ y, const PeerAr ar) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const unsigned e = unsigned(*ar.epoch) + 1u;
    const int par = int(e & 1u);
    const int per = ar.n / kArBlocks;
    for (int i = threadIdx.x; i < per; i += blockDim.x) {
        const int row = blockIdx.x * per + i;
        const unsigned long long w = tag_word(e, y[row]);
        for (int r = 0; r < ar.world; ++r) st_word(ar.slots[r] + (size_t(par) * ar.world + ar.rank) * ar.n + row, w);
    }
}

// The same exchange as a plain in-place all-reduce of count fp32 values
// (p100_tp_allreduce_sum over peer memory): thread t of CTA b owns values
// 4 (256 b + t) .. +3.  It pushes them to every rank as tagged words, waits
// (bounded) until its own arena holds every rank's words of this epoch, and
// writes their sum in rank order (every rank gets the same bits).  The CTAs
// read the epoch when they start; the last one to finish (ticket) advances
// it.  A wait that runs out (ar.wait_ns: ranks may reach a collective far
// apart, so the caller gives a long limit) marks the exchange broken in
// *broken, and every later call gives up at once instead of waiting again
// (its epochs no longer match the other ranks').  Grid ceil(count / 1024) x
// 256 with count <= ar.n.  Every thread pushes before it waits, so no wait
// depends on a CTA of this grid that has not started.
constexpr int kArThreads = 256;
__device__ __forceinline__ void st_words2(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(float* __restrict__ buf, int count, const PeerAr ar,
                                                                    int* __restrict__ ticket, int* __restrict__ broken) {
    // launched as a programmatic dependent: buf (and the epoch) are read
    // only after the previous kernel has ended
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const unsigned e = unsigned(*ar.epoch) + 1u;
    const int par = int(e & 1u);
    const int i0 = (blockIdx.x * kArThreads + threadIdx.x) * 4;
    bool timed_out = *reinterpret_cast<volatile int*>(broken) != 0;
    if (i0 < count) {
        const int m = min(4, count - i0);
        unsigned long long w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = tag_word(e, j < m ? buf[i0 + j] : 0.f);
        for (int r = 0; r < ar.world; ++r) {
            unsigned long long* dst = ar.slots[r] + (size_t(par) * ar.world + ar.rank) * ar.n + i0;
            st_words2(dst, w[0], w[1]);
            st_words2(dst + 2, w[2], w[3]);
        }
        const unsigned long long* base = ar.slots[ar.rank] + size_t(par) * ar.world * ar.n + i0;
        const unsigned long long limit = ar.wait_ns ? ar.wait_ns : kWaitLimitNs;
        unsigned long long start = 0;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < ar.world && !timed_out; ++r) {
            unsigned long long a, b, c, d;
            for (;;) {
                ld_words2(base + size_t(r) * ar.n, a, b);
                ld_words2(base + size_t(r) * ar.n + 2, c, d);
                if (unsigned(a >> 32) == e && unsigned(b >> 32) == e && unsigned(c >> 32) == e &&
                    unsigned(d >> 32) == e)
                    break;
                const unsigned long long now = globaltimer_ns();
                if (!start) {
                    start = now;
                } else if (now - start > limit) {
                    timed_out = true;
                    break;
                }
            }
            const float f[4] = {__uint_as_float(uint32_t(a)), __uint_as_float(uint32_t(b)), __uint_as_float(uint32_t(c)),
                                __uint_as_float(uint32_t(d))};
#pragma unroll
            for (int j = 0; j < 4; ++j) s[j] = r == 0 ? f[j] : __fadd_rn(s[j], f[j]);
        }
        if (!timed_out)
            for (int j = 0; j < m; ++j) buf[i0 + j] = s[j];
    }
    if (timed_out) {
        atomicExch(&g_device_error, kDevErrTimeout);
        atomicExch(broken, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ticket, 1) == int(gridDim.x) - 1) {
            *ticket = 0;
            *ar.epoch = int(e);   // read by the next call, which starts after this kernel ends
        }
    }
}

// ------------------------------------------------------------------ RMSNorm
// Q8_1 block of 32 values held four per lane by 8 consecutive lanes (lane j
// of the octet holds elements 4j..4j+3 in v[0..3]).  Same bytes as
// warp_q8_1_block: the 32-lane XOR butterfly (16, 8, 4, 2, 1) pairs element
// 4j+e with 4(j^4)+e, 4(j^2)+e, 4(j^1)+e, then 4j+(e^2), 4j+(e^1), which is
// lanes 4, 2, 1 apart and then inside the lane; max is order-free.
__device__ __forceinline__ void octet_q8_1_block(const float (&v)[4], int j, uint8_t* blk) {
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    float s[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
    for (int off = 4; off > 0; off >>= 1)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[e] = __fadd_rn(s[e], __shfl_xor_sync(0xffffffffu, s[e], off));
    const float s2 = __fadd_rn(s[0], s[2]), s3 = __fadd_rn(s[1], s[3]);
    const float sum = __fadd_rn(s2, s3);
    const float d = amax / 127.0f;
    uint32_t codes = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int q = amax == 0.0f ? 0 : static_cast<int>(roundf(v[e] / d));
        codes |= uint32_t(uint8_t(static_cast<int8_t>(q))) << (8 * e);
    }
    if (!blk) return;
    if (j == 0) {
        const uint32_t ds = uint32_t(__half_as_ushort(__float2half_rn(d))) |
                            (uint32_t(__half_as_ushort(__float2half_rn(sum))) << 16);
        *reinterpret_cast<uint32_t*>(blk) = ds;
    }
    *reinterpret_cast<uint32_t*>(blk + 4 + 4 * j) = codes;
}

// x[i] += delta[i] (when delta), then ss = sum x[i]^2 in the fixed order
//   thread t owns the float4 chunks c = t, t + 1024, ... (elements 4c..4c+3):
//   s_t = fma(x, x, s_t) over its chunks ascending, the 4 elements in order;
//   warp: XOR butterfly 16,8,4,2,1; block: ((w0 + w1) + ...) + w31;
// r = 1 / sqrt(ss / k + eps) (IEEE sqrt and divisions);
// y[i] = (x[i] * r) * w[i], quantised to Q8_1 per 32: block b is chunks
// 8b..8b+7, held by one octet of lanes of one warp.  y_out optional.
// One block per batch row; k % 32 == 0 and k <= kNormMaxK.
constexpr int kNormChunks = 4;    // float4 chunks per thread at most
constexpr int kNormMaxK = kNormChunks * kNormThreads * 4;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_q8_1_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                                  const float* __restrict__ w, float eps, int k,
                                                                  uint8_t* __restrict__ xq, float* __restrict__ y_out,
                                                                  const PeerAr ar) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    __shared__ float s_part[kNormThreads / 32];
    __shared__ float s_r;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4* xr = reinterpret_cast<float4*>(x + size_t(blockIdx.x) * k);
    const float4* dr = delta ? reinterpret_cast<const float4*>(delta + size_t(blockIdx.x) * k) : nullptr;
    const int nc = k / 4;
    float4 v[kNormChunks];
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
        const int c = tid + i * kNormThreads;
        v[i] = c < nc ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (dr) {
#pragma unroll
        for (int i = 0; i < kNormChunks; ++i) {
            const int c = tid + i * kNormThreads;
            if (c < nc) {
                const float4 d4 = dr[c];
                v[i] = make_float4(__fadd_rn(v[i].x, d4.x), __fadd_rn(v[i].y, d4.y), __fadd_rn(v[i].z, d4.z),
                                   __fadd_rn(v[i].w, d4.w));
                xr[c] = v[i];
            }
        }
    } else if (ar.world > 0) {
        // delta = the peer all-reduce of this epoch (batch 1, n = k): every
        // thread polls the tagged words of its own chunks (rows 4c..4c+3 of
        // every rank), bounded, then adds the ranks in order
        const unsigned e = unsigned(*ar.epoch) + 1u;
        const int par = int(e & 1u);
        const unsigned long long* base = ar.slots[ar.rank] + size_t(par) * ar.world * ar.n;
        const unsigned long long limit = ar.wait_ns ? ar.wait_ns : kWaitLimitNs;
        const unsigned long long start = globaltimer_ns();
        bool ok = true;
#pragma unroll
        for (int i = 0; i < kNormChunks; ++i) {
            const int c = tid + i * kNormThreads;
            if (c >= nc) continue;
            float4 d4 = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < ar.world; ++r) {
                const unsigned long long* wp = base + size_t(r) * ar.n + 4 * c;
                unsigned long long w0, w1, w2, w3;
                for (;;) {
                    ld_words2(wp, w0, w1);
                    ld_words2(wp + 2, w2, w3);
                    if (unsigned(w0 >> 32) == e && unsigned(w1 >> 32) == e && unsigned(w2 >> 32) == e &&
                        unsigned(w3 >> 32) == e)
                        break;
                    if (!ok || globaltimer_ns() - start > limit) {
                        ok = false;
                        break;
                    }
                }
                const float4 o = make_float4(__uint_as_float(unsigned(w0)), __uint_as_float(unsigned(w1)),
                                             __uint_as_float(unsigned(w2)), __uint_as_float(unsigned(w3)));
                d4 = r == 0 ? o
                            : make_float4(__fadd_rn(d4.x, o.x), __fadd_rn(d4.y, o.y), __fadd_rn(d4.z, o.z),
                                          __fadd_rn(d4.w, o.w));
            }
            v[i] = make_float4(__fadd_rn(v[i].x, d4.x), __fadd_rn(v[i].y, d4.y), __fadd_rn(v[i].z, d4.z),
                               __fadd_rn(v[i].w, d4.w));
            xr[c] = v[i];
        }
        if (!__syncthreads_and(ok) && tid == 0) atomicExch(&g_device_error, kDevErrTimeout);
        if (tid == 0) *ar.epoch = int(e);   // read by the next push and reduce, which start after this kernel ends
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
        const int c = tid + i * kNormThreads;
        if (c < nc) {
            s = fmaf(v[i].x, v[i].x, s);
            s = fmaf(v[i].y, v[i].y, s);
            s = fmaf(v[i].z, v[i].z, s);
            s = fmaf(v[i].w, v[i].w, s);
        }
    }
    s = warp_sum(s);
    if (lane == 0) s_part[warp] = s;
    __syncthreads();
    if (tid == 0) {
        float t = s_part[0];
        for (int i = 1; i < kNormThreads / 32; ++i) t = __fadd_rn(t, s_part[i]);
        s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, float(k)), eps)));
    }
    __syncthreads();
    const float r = s_r;
    const float4* w4 = reinterpret_cast<const float4*>(w);
    uint8_t* qrow = xq + size_t(blockIdx.x) * (k / 32) * 36;
    float4* yr = y_out ? reinterpret_cast<float4*>(y_out + size_t(blockIdx.x) * k) : nullptr;
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
        if (i * kNormThreads >= nc) break;   // uniform over the block
        // every lane runs the octet quantiser (its shuffles need the whole
        // warp); lanes past the row's end quantise zeros and store nothing
        const int c = tid + i * kNormThreads;
        const bool live = c < nc;
        const float4 wv = live ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float y[4] = {__fmul_rn(__fmul_rn(v[i].x, r), wv.x), __fmul_rn(__fmul_rn(v[i].y, r), wv.y),
                            __fmul_rn(__fmul_rn(v[i].z, r), wv.z), __fmul_rn(__fmul_rn(v[i].w, r), wv.w)};
        if (live && yr) yr[c] = make_float4(y[0], y[1], y[2], y[3]);
        octet_q8_1_block(y, c & 7, live ? qrow + size_t(c >> 3) * 36 : nullptr);
    }
}

// --------------------------------------------------------- RoPE + KV append
// qkv = [q heads | k heads | v heads] x head_dim fp32 (the fused QKV mat-vec
// output).  Adjacent-pair rotation (llama.cpp's "norm" RoPE for Llama):
//   (x0, x1) at (2i, 2i+1) -> (x0 c - x1 s, x0 s + x1 c),  (c, s) = cs[pos][i]
// with cs from a host table (cos/sin of pos * theta^(-2i/d), computed in
// double).  q is rotated in place; rotated k and plain v are rounded to fp16
// (nearest) into the caches at row pos: cache[(head * head_stride) + pos*d].
// Grid: one block per head (q, k and v heads), head_dim / 2 threads.
__global__ void rope_kv_append_kernel(float* __restrict__ qkv, int nq, int nkv, int hd, const float2* __restrict__ cs,
                                      int max_pos, const int* __restrict__ pos_dev, __half* __restrict__ kc,
                                      __half* __restrict__ vc, long long head_stride) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const int pos = *pos_dev;
    if (pos < 0 || pos >= max_pos) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(&g_device_error, kDevErrInput);
        return;
    }
    const int h = blockIdx.x, i = threadIdx.x;   // pair i of head h
    float* v = qkv + size_t(h) * hd + 2 * i;
    const float x0 = v[0], x1 = v[1];
    if (h >= nq + nkv) {   // v head
        __half2* dst = reinterpret_cast<__half2*>(vc + (h - nq - nkv) * head_stride + size_t(pos) * hd + 2 * i);
        *dst = __halves2half2(__float2half_rn(x0), __float2half_rn(x1));
        return;
    }
    const float2 t = cs[size_t(pos) * (hd / 2) + i];
    const float y0 = __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
    const float y1 = __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x));
    if (h < nq) {
        v[0] = y0;
        v[1] = y1;
    } else {
        __half2* dst = reinterpret_cast<__half2*>(kc + (h - nq) * head_stride + size_t(pos) * hd + 2 * i);
        *dst = __halves2half2(__float2half_rn(y0), __float2half_rn(y1));
    }
}

// ------------------------------------------------------------ SwiGLU + Q8_1
// exp(x) for x in [-104, 89]: n = rint(x / ln2), r = (x - n ln2_hi) - n ln2_lo
// (Cody-Waite, ln2 split so n * ln2_hi is exact), e^r by its Taylor series to
// degree 8 in Horner form (|r| <= 0.347: truncation < 1.3e-10 relative), then
// scaled by 2^n in two steps (so 2^n itself never overflows or flushes).
// Below -104 the result is 0, above 89 +inf.
__device__ __forceinline__ float dec_exp(float x) {
    if (x < -104.0f) return 0.0f;
    if (x > 89.0f) return __int_as_float(0x7f800000);
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    const float r = fmaf(-n, 1.42860677e-06f, fmaf(-n, 0.693145751953125f, x));
    float p = 2.48015873e-05f;              // 1/8!
    p = fmaf(p, r, 1.98412698e-04f);        // 1/7!
    p = fmaf(p, r, 1.38888889e-03f);        // 1/6!
    p = fmaf(p, r, 8.33333333e-03f);        // 1/5!
    p = fmaf(p, r, 4.16666667e-02f);        // 1/4!
    p = fmaf(p, r, 1.66666667e-01f);        // 1/3!
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = static_cast<int>(n);
    const int n1 = ni / 2, n2 = ni - n1;
    return __fmul_rn(__fmul_rn(p, __int_as_float((n1 + 127) << 23)), __int_as_float((n2 + 127) << 23));
}

// h = silu(g) * u = (g / (1 + exp(-g))) * u, gate_up row = [g(n) | u(n)];
// h quantised to Q8_1 per 32.  Grid: (n / 256 rounded up, batch); n % 32 == 0.
__global__ void __launch_bounds__(256) swiglu_q8_1_kernel(const float* __restrict__ gu, int n,
                                                         uint8_t* __restrict__ xq) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    if (b >= n / 32) return;
    const float* row = gu + size_t(blockIdx.y) * 2 * n;
    const int i = b * 32 + lane;
    const float g = row[i], u = row[n + i];
    const float silu = __fdiv_rn(g, __fadd_rn(1.0f, dec_exp(-g)));
    warp_q8_1_block(__fmul_rn(silu, u), lane, xq + (size_t(blockIdx.y) * (n / 32) + b) * 36);
}

// ----------------------------------------------------------------- argmax
// Index of the largest value (lowest index among equal ones; NaN never wins;
// an all-NaN or empty row gives index 0, value -inf).
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// One block: the row's argmax to idx_out/val_out.  If advance is set, also
// the decode step's bookkeeping: *token = argmax + index_base, *pos += 1.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ x, int n, int index_base,
                                                              int* __restrict__ idx_out, float* __restrict__ val_out,
                                                              int* __restrict__ token, int* __restrict__ pos) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    __shared__ float s_v[kArgmaxThreads / 32];
    __shared__ int s_i[kArgmaxThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* row = x + size_t(blockIdx.x) * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += kArgmaxThreads) {
        const float v = row[i];
        if (better(v, i, bv, bi)) { bv = v; bi = i; }   // NaN compares false
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w)
            if (better(s_v[w], s_i[w], bv, bi)) { bv = s_v[w]; bi = s_i[w]; }
        if (bi == 0x7fffffff) bi = 0;
        if (idx_out) idx_out[blockIdx.x] = bi + index_base;
        if (val_out) val_out[blockIdx.x] = bv;
        if (token) *token = bi + index_base;
        if (pos) *pos += 1;
    }
}

// The best of per-rank (value, index) candidates laid out [rank][2] as
// floats (indices below 2^24 are exact), then the step's bookkeeping.
__global__ void pick_candidates_kernel(const float* __restrict__ cand, int n, int* __restrict__ token,
                                       int* __restrict__ pos) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    if (threadIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < n; ++r) {
        const float v = cand[2 * r];
        const int i = static_cast<int>(cand[2 * r + 1]);
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    *token = bi == 0x7fffffff ? 0 : bi;
    *pos += 1;
}

// Local argmax as a (value, global index) pair of floats, for the all-gather.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_pair_kernel(const float* __restrict__ x, int n, int index_base,
                                                                   float* __restrict__ pair) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    __shared__ float s_v[kArgmaxThreads / 32];
    __shared__ int s_i[kArgmaxThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += kArgmaxThreads) {
        const float v = x[i];
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w)
            if (better(s_v[w], s_i[w], bv, bi)) { bv = s_v[w]; bi = s_i[w]; }
        pair[0] = bv;
        pair[1] = float(bi == 0x7fffffff ? index_base : bi + index_base);
    }
}

// -------------------------------------------------------------- embedding
// x = dequantised row *token of the embedding matrix (one thread per slab).
template <int TYPE>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t* __restrict__ emb, size_t row_bytes, int vocab,
                                                    int hidden, const int* __restrict__ token, float* __restrict__ x) {
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= hidden / 32) return;
    const int t = *token;
    if (t < 0 || t >= vocab) {
        if (j == 0) atomicExch(&g_device_error, kDevErrInput);
        return;
    }
    float vals[32];
    dequant_slab<TYPE>(emb + size_t(t) * row_bytes, j, vals);
    float4* dst = reinterpret_cast<float4*>(x + size_t(j) * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
}

// ------------------------------------------------- synthetic initialisation
// Counter-based: every value is a function of (seed, tensor id, global
// coordinates), so a tensor-parallel slice initialised on its own rank holds
// exactly the rows/blocks the unsplit tensor holds there.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {   // splitmix64 finaliser
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float unit_float(uint64_t h) {   // (0, 1)
    return (float(uint32_t(h >> 40)) + 0.5f) * (1.0f / 16777216.0f);
}
__device__ __forceinline__ float normal_from(uint64_t h) {   // Box-Muller
    const float u1 = unit_float(h), u2 = unit_float(mix64(h));
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}
__device__ __forceinline__ void store_half(uint8_t* p, float v) { store_half_bits(p, v); }

// Weight blocks of a rows x blocks matrix slice whose (row, block) (0, 0)
// sits at global (row0, block0).  Q4_0: d = |N(0,1)| * dscale, codes
// U{0..15}; Q8_0: d likewise, codes U{-127..127}; Q4_K and Q5_K: d and dmin
// |N| * dscale, scale bytes and code bits uniform; Q6_K: ql, qh and the
// int8 sub-block scales uniform, d = |N| * dscale.  Each format's d (and
// dmin) is then divided by the power of two nearest to the RMS of its values
// over Q4_0's under these draws (measured: 16, 69, 144 and 309 for Q8_0,
// Q4_K, Q5_K and Q6_K), so a model whose tensors mix formats keeps one
// scale.  One thread per block.
template <int TYPE>
__global__ void init_weights_kernel(uint8_t* __restrict__ w, size_t row_bytes, int rows, int blocks, uint64_t key,
                                    long long row0, long long block0, float dscale) {
    const long long id = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= static_cast<long long>(rows) * blocks) return;
    const int r = static_cast<int>(id / blocks), b = static_cast<int>(id % blocks);
    const uint64_t h = mix64(key ^ mix64((uint64_t(row0 + r) << 24) ^ uint64_t(block0 + b)));
    constexpr int kBytes = TYPE == P100_Q4_0 ? 18
                           : TYPE == P100_Q8_0 ? 34
                           : TYPE == P100_Q4_K ? 144
                           : TYPE == P100_Q5_K ? 176
                                               : 210;
    uint8_t* blk = w + size_t(r) * row_bytes + size_t(b) * kBytes;
    constexpr float kFormat = TYPE == P100_Q4_0   ? 1.0f
                              : TYPE == P100_Q8_0 ? 1.0f / 16
                              : TYPE == P100_Q4_K ? 1.0f / 64
                              : TYPE == P100_Q5_K ? 1.0f / 128
                                                  : 1.0f / 256;
    dscale *= kFormat;   // a power of two: exact
    uint64_t z = mix64(h ^ 0x5bd1e995ull);
    if (TYPE == P100_Q6_K) {
        for (int i = 0; i < 208; ++i) {   // ql[128], qh[64], scales[16]
            if ((i & 7) == 0) z = mix64(z);
            blk[i] = uint8_t(z >> (8 * (i & 7)));
        }
        store_half(blk + 208, fabsf(normal_from(h)) * dscale);
        return;
    }
    store_half(blk, fabsf(normal_from(h)) * dscale);
    if (TYPE == P100_Q4_K || TYPE == P100_Q5_K) {
        store_half(blk + 2, fabsf(normal_from(z)) * dscale);
        for (int i = 4; i < kBytes; ++i) {
            if ((i & 7) == 4) z = mix64(z);
            blk[i] = uint8_t(z >> (8 * (i & 7)));
        }
    } else if (TYPE == P100_Q4_0) {
        for (int i = 2; i < kBytes; ++i) {
            if ((i & 7) == 2) z = mix64(z);
            blk[i] = uint8_t(z >> (8 * (i & 7)));
        }
    } else {
        for (int i = 2; i < kBytes; ++i) {
            z = mix64(z);
            blk[i] = uint8_t(static_cast<int8_t>(int(z % 255u) - 127));
        }
    }
}

// fp32 vector: lo + (hi - lo) * U(0,1) at global index base + i.
__global__ void init_uniform_kernel(float* __restrict__ v, long long n, uint64_t key, long long base, float lo,
                                    float hi) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    v[i] = lo + (hi - lo) * unit_float(mix64(key ^ uint64_t(base + i)));
}

// fp16 KV rows [0, npos) of `heads` heads with stride head_stride:
// N(0,1) * scale at global (head0 + h, pos, dim).
__global__ void init_kv_kernel(__half* __restrict__ c, int heads, int npos, int hd, long long head_stride,
                               uint64_t key, int head0, float scale) {
    const long long id = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long per_head = static_cast<long long>(npos) * hd;
    if (id >= per_head * heads) return;
    const int h = static_cast<int>(id / per_head);
    const long long e = id % per_head;
    const uint64_t g = (uint64_t(head0 + h) << 40) ^ uint64_t(e);
    c[h * head_stride + e] = __float2half_rn(normal_from(mix64(key ^ mix64(g))) * scale);
}

// The same values as init_kv_kernel (before its fp16 rounding), quantised
// to q8_0 / q4_0 blocks with kvq::quantize_block_warp: one warp per block,
// lane = value; row (h, pos) at c + (h * max_ctx + pos) * hd/32 blocks.
template <int KV>
__global__ void init_kv_quant_kernel(uint8_t* __restrict__ c, int heads, int npos, int hd, int max_ctx, uint64_t key,
                                     int head0, float scale) {
    const long long blk = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long long per_head = static_cast<long long>(npos) * (hd / 32);
    if (blk >= per_head * heads) return;   // warp-uniform
    const int h = static_cast<int>(blk / per_head);
    const long long e = (blk % per_head) * 32 + lane;   // value index within the head's rows
    const uint64_t g = (uint64_t(head0 + h) << 40) ^ uint64_t(e);
    const float x = normal_from(mix64(key ^ mix64(g))) * scale;
    const long long pos = e / hd;
    uint8_t* row = c + (static_cast<long long>(h) * max_ctx + pos) * (hd / 32) * kvq::block_bytes<KV>();
    kvq::quantize_block_warp<KV>(x, lane, row + ((e % hd) / 32) * kvq::block_bytes<KV>());
}

}  // namespace dec
}  // namespace p100b
