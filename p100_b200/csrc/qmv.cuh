// qmv.cuh — quantised mat-vec y = W x for Q4_0 / Q8_0 / Q4_K (and, on the
// generic kernel only, Q5_K / Q6_K) weights against
// Q8_1 activations, batch 1..16, on CUDA cores (int8 dp4a).
//
// Bulk path (16-byte aligned rows, k % 256 == 0), warp-specialised:
//   * Each CTA owns a contiguous, balanced range of rows; its weight bytes are
//     one contiguous span of the matrix, cut into stages of R whole rows of
//     about 16 KB (smaller bulk copies lose bandwidth).
//   * One producer warp streams the stages HBM -> shared memory with untiled
//     bulk-async copies (cp.async.bulk, L2 evict-first) into a ring of slots,
//     each with a "full" and an "empty" mbarrier.
//   * All eight consumer warps work on every stage, in order: the stage's
//     R x (k/64) items (64 weights each: two Q4_0/Q8_0 blocks, or a quarter
//     Q4_K super-block) are split into eight contiguous shares, so a stage is
//     held only briefly and most of the ring stays in flight.  A share spans
//     at most two rows; each warp finishes its partial row sums with an XOR
//     butterfly and stores them.  The last warp to finish a stage (a shared-
//     memory ticket picks it) adds the eight partials of each row in warp
//     order, writes y and frees the slot.  The ticket decides who adds, never
//     the order, so results are deterministic.
//   * The activations are staged once per CTA in shared memory with the int8
//     codes transposed (word i of every block contiguous), so a lane's 8-byte
//     reads of its block pair are bank-conflict free.
//   * For one column the CTA keeps to half an SM, so two launches of a chain
//     (programmatic dependent launch) are resident together: the next one's
//     weights stream in while this one finishes.
//
// The per-block arithmetic is that of qmv::evaluate's q81 path
// (qmv_model.cpp:147-180): exact int32 block dots, then FP32 scaling with the
// fp16 scales.  Only the FP32 summation order across blocks differs from the
// sequential CPU model.
#pragma once
#include "common.cuh"
#include "quant.cuh"

namespace p100b {
namespace qmv {

constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;   // 8 consumer warps + 1 producer warp
constexpr int kMaxSlots = 16;
constexpr int kMaxRows = 8;                       // rows per stage
constexpr int kSmemLimit = 227 * 1024;

// Activation operands of one item (blocks A = 2*it and B = 2*it+1) for one column.
struct ItemAct {
    int q[16];   // int8 codes: A words 0..7, then B words 0..7
    float4 m;    // (dA, mA, dB, mB): m = fp16 sum of x (Q4_0), sum of codes (Q4_K), 0 (Q8_0)
};

struct Params {
    const uint8_t* w;
    const uint8_t* xq;     // block_q8_1 rows, 36 bytes per 32 values
    float* y;
    int rows, k;
    int col0;              // first activation column of this launch
    int row_bytes;
    int ipr;               // items per row = k / 64
    int rps;               // rows per stage (1..kMaxRows)
    int nslot;
    int slot_bytes;        // ring slot stride (multiple of 128)
    int part_off, codes_off, meta_off, ring_off;   // shared-memory offsets
};

// Adds item `it` of one staged row to acc[c] for every column c.
template <int TYPE, int B>
__device__ __forceinline__ void item_dot(const uint8_t* __restrict__ row, int it, const ItemAct (&a)[B],
                                         float (&acc)[B]) {
    if (TYPE == P100_Q4_0) {
        // 36 bytes: block A at +0 (d, 16 nibble bytes at +2), block B at +18.
        const uint32_t* p = reinterpret_cast<const uint32_t*>(row + it * 36);
        uint32_t W[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) W[i] = p[i];
        const float dA = half_lo(W[0]), dB = half_hi(W[4]);
        uint32_t qa[4], qb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qa[i] = shift2(W[i], W[i + 1]);
            qb[i] = W[5 + i];
        }
#pragma unroll
        for (int c = 0; c < B; ++c) {
            int sa0 = 0, sa1 = 0, sb0 = 0, sb1 = 0;   // four independent dp4a chains
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // byte m: low nibble is element m, high nibble element m+16
                sa0 = __dp4a(static_cast<int>(qa[i] & 0x0f0f0f0fu), a[c].q[i], sa0);
                sa1 = __dp4a(static_cast<int>((qa[i] >> 4) & 0x0f0f0f0fu), a[c].q[4 + i], sa1);
                sb0 = __dp4a(static_cast<int>(qb[i] & 0x0f0f0f0fu), a[c].q[8 + i], sb0);
                sb1 = __dp4a(static_cast<int>((qb[i] >> 4) & 0x0f0f0f0fu), a[c].q[12 + i], sb1);
            }
            // d_w * (d_x * sum(nib*q) - 8 * sum(x)): the -8 offset through the
            // block sum, as the q81 path does per half block.
            acc[c] = fmaf(dA, fmaf(float(sa0 + sa1), a[c].m.x, -8.0f * a[c].m.y), acc[c]);
            acc[c] = fmaf(dB, fmaf(float(sb0 + sb1), a[c].m.z, -8.0f * a[c].m.w), acc[c]);
        }
    } else if (TYPE == P100_Q8_0) {
        // 68 bytes: block A at +0 (codes at +2), block B at +34 (codes at +36).
        const uint32_t* p = reinterpret_cast<const uint32_t*>(row + it * 68);
        uint32_t W[17];
#pragma unroll
        for (int i = 0; i < 17; ++i) W[i] = p[i];
        const float dA = half_lo(W[0]), dB = half_hi(W[8]);
        int qa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) qa[i] = static_cast<int>(shift2(W[i], W[i + 1]));
#pragma unroll
        for (int c = 0; c < B; ++c) {
            int sa0 = 0, sa1 = 0, sb0 = 0, sb1 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                sa0 = __dp4a(qa[i], a[c].q[i], sa0);
                sa1 = __dp4a(qa[4 + i], a[c].q[4 + i], sa1);
                sb0 = __dp4a(static_cast<int>(W[9 + i]), a[c].q[8 + i], sb0);
                sb1 = __dp4a(static_cast<int>(W[13 + i]), a[c].q[12 + i], sb1);
            }
            acc[c] = fmaf(dA * a[c].m.x, float(sa0 + sa1), acc[c]);
            acc[c] = fmaf(dB * a[c].m.z, float(sb0 + sb1), acc[c]);
        }
    } else {
        // Quarter super-block: header (d, dmin, 12 scale bytes) + 32 nibble
        // bytes holding sub-blocks 2*qq (low nibbles) and 2*qq+1 (high).
        const int sbk = it >> 2, qq = it & 3;
        const uint8_t* sb = row + sbk * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(sb);
        const uint4 n0 = *reinterpret_cast<const uint4*>(sb + 16 + qq * 32);
        const uint4 n1 = *reinterpret_cast<const uint4*>(sb + 32 + qq * 32);
        const float d = half_lo(hdr.x), dmin = half_hi(hdr.x);
        // Six-bit scales/mins of sub-blocks 2qq and 2qq+1 straight from the
        // packed words (bytes 0-3: hdr.y, 4-7: hdr.z, 8-11: hdr.w), the
        // get_scale_min_k4 rule of qmv_model.cpp:72-77.
        int sc0, mn0, sc1, mn1;
        if (qq < 2) {
            const int sh0 = 16 * qq, sh1 = sh0 + 8;              // bytes j, j < 4
            sc0 = (hdr.y >> sh0) & 63;
            mn0 = (hdr.z >> sh0) & 63;
            sc1 = (hdr.y >> sh1) & 63;
            mn1 = (hdr.z >> sh1) & 63;
        } else {
            const int sh0 = 16 * (qq - 2), sh1 = sh0 + 8;        // j - 4 in 0..3
            sc0 = ((hdr.w >> sh0) & 15) | (((hdr.y >> (sh0 + 6)) & 3) << 4);
            mn0 = ((hdr.w >> (sh0 + 4)) & 15) | (((hdr.z >> (sh0 + 6)) & 3) << 4);
            sc1 = ((hdr.w >> sh1) & 15) | (((hdr.y >> (sh1 + 6)) & 3) << 4);
            mn1 = ((hdr.w >> (sh1 + 4)) & 15) | (((hdr.z >> (sh1 + 6)) & 3) << 4);
        }
        const uint32_t N[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
        for (int c = 0; c < B; ++c) {
            int s0a = 0, s0b = 0, s1a = 0, s1b = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                s0a = __dp4a(static_cast<int>(N[i] & 0x0f0f0f0fu), a[c].q[i], s0a);
                s0b = __dp4a(static_cast<int>(N[4 + i] & 0x0f0f0f0fu), a[c].q[4 + i], s0b);
                s1a = __dp4a(static_cast<int>((N[i] >> 4) & 0x0f0f0f0fu), a[c].q[8 + i], s1a);
                s1b = __dp4a(static_cast<int>((N[4 + i] >> 4) & 0x0f0f0f0fu), a[c].q[12 + i], s1b);
            }
            // d * sum_j dx_j*(dot_j*sc_j) - dmin * sum_j dx_j*(sumq_j*mn_j)
            // (qmv_model.cpp:175-178, summed over both sub-blocks)
            const float sd = fmaf(a[c].m.x, float((s0a + s0b) * sc0), a[c].m.z * float((s1a + s1b) * sc1));
            const float sm = fmaf(a[c].m.x, a[c].m.y * float(mn0), a[c].m.z * (a[c].m.w * float(mn1)));
            acc[c] = fmaf(d, sd, acc[c]);
            acc[c] = fmaf(-dmin, sm, acc[c]);
        }
    }
}

template <int TYPE, int B>
__global__ void __launch_bounds__(kThreads, B == 1 ? 2 : 1) qmv_bulk_kernel(const Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    unsigned* ticket = reinterpret_cast<unsigned*>(empty + kMaxSlots);          // [kMaxSlots]
    float* partial = reinterpret_cast<float*>(smem + p.part_off);              // [slot][warp][row][col]
    uint32_t* codes = reinterpret_cast<uint32_t*>(smem + p.codes_off);         // [B][8][nb] words
    float2* meta = reinterpret_cast<float2*>(smem + p.meta_off);               // [B][nb]
    uint8_t* ring = smem + p.ring_off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = p.k / 32;
    const int r0 = static_cast<int>(static_cast<long long>(p.rows) * blockIdx.x / gridDim.x);
    const int r1 = static_cast<int>(static_cast<long long>(p.rows) * (blockIdx.x + 1) / gridDim.x);
    const int nst = (r1 - r0 + p.rps - 1) / p.rps;

    if (tid == 0) {
        for (int s = 0; s < p.nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            ticket[s] = 0;
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_allow_dependents();

    if (warp == kConsumers) {
        // ---- producer: weights never depend on the previous kernel
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            for (int s = 0; s < nst; ++s) {
                const int slot = s % p.nslot;
                if (s >= p.nslot && !mbar_wait(&empty[slot], ((s / p.nslot) - 1) & 1)) break;
                const int first = r0 + s * p.rps;
                const uint32_t bytes = static_cast<uint32_t>(min(p.rps, r1 - first)) * p.row_bytes;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load(ring + size_t(slot) * p.slot_bytes, p.w + size_t(first) * p.row_bytes, bytes, &full[slot],
                          policy);
            }
        }
        return;
    }

    // ---- consumers: stage this launch's Q8_1 activations (they may come from
    // the previous kernel), codes transposed.
    pdl_wait_prior_grid();
    for (int idx = tid; idx < B * nb; idx += kConsumers * 32) {
        const int c = idx / nb, j = idx % nb;
        const uint32_t* blk = reinterpret_cast<const uint32_t*>(p.xq + (size_t(p.col0 + c) * nb + j) * 36);
        const uint32_t ds = __ldg(blk);
        int sumq = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t wq = __ldg(blk + 1 + i);
            codes[(c * 8 + i) * nb + j] = wq;
            sumq = __dp4a(static_cast<int>(wq), 0x01010101, sumq);
        }
        const float m = TYPE == P100_Q4_0 ? half_hi(ds) : TYPE == P100_Q4_K ? float(sumq) : 0.f;
        meta[c * nb + j] = make_float2(half_lo(ds), m);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");

    for (int s = 0; s < nst; ++s) {
        const int slot = s % p.nslot;
        // A timed-out wait is decided for the whole warp (vote), so no lane is
        // left in a shuffle its peers have abandoned.
        if (!__all_sync(0xffffffffu, mbar_wait(&full[slot], (s / p.nslot) & 1))) break;
        const uint8_t* stage = ring + size_t(slot) * p.slot_bytes;
        const int first = r0 + s * p.rps;
        const int nr = min(p.rps, r1 - first);
        // This warp's share of the stage's nr x ipr items: at most two rows.
        const int n_items = nr * p.ipr;
        const int f0 = n_items * warp / kConsumers, f1 = n_items * (warp + 1) / kConsumers;
        const int rw = f0 / p.ipr;   // first row of the share
        float acc[2][B];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < B; ++c) acc[h][c] = 0.f;
        for (int f = f0 + lane; f < f1; f += 32) {
            const int r = f / p.ipr, it = f - r * p.ipr;
            ItemAct a[B];
#pragma unroll
            for (int c = 0; c < B; ++c) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint2 v = *reinterpret_cast<const uint2*>(codes + (c * 8 + i) * nb + 2 * it);
                    a[c].q[i] = static_cast<int>(v.x);
                    a[c].q[8 + i] = static_cast<int>(v.y);
                }
                a[c].m = *reinterpret_cast<const float4*>(meta + c * nb + 2 * it);
            }
            float tmp[B];
#pragma unroll
            for (int c = 0; c < B; ++c) tmp[c] = 0.f;
            item_dot<TYPE, B>(stage + size_t(r) * p.row_bytes, it, a, tmp);
            const bool second = r != rw;
#pragma unroll
            for (int c = 0; c < B; ++c) {
                acc[0][c] += second ? 0.f : tmp[c];
                acc[1][c] += second ? tmp[c] : 0.f;
            }
        }
        float v[2][B];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < B; ++c) v[h][c] = warp_sum(acc[h][c]);
        // partial[slot][warp][row][col]: this warp's sums, zero off its share.
        float* mine = partial + (size_t(slot) * kConsumers + warp) * (kMaxRows * B);
        if (lane < nr * B) {
            const int r = lane / B, c = lane % B;
            float out = 0.f;
#pragma unroll
            for (int cc = 0; cc < B; ++cc)
                if (cc == c) out = r == rw ? v[0][cc] : r == rw + 1 ? v[1][cc] : 0.f;
            mine[lane] = out;
        }
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&ticket[slot], 1u) == kConsumers - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __syncwarp();
            __threadfence_block();
            if (lane < nr * B) {
                const int r = lane / B, c = lane % B;
                const float* base = partial + size_t(slot) * kConsumers * (kMaxRows * B) + lane;
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumers; ++w) sum += base[w * (kMaxRows * B)];
                p.y[size_t(p.col0 + c) * p.rows + first + r] = sum;
            }
            __syncwarp();
            if (lane == 0) {
                ticket[slot] = 0;
                mbar_arrive(&empty[slot]);
            }
        }
    }
}

// ------------------------------------------------------------------ generic
// Any 2-byte aligned matrix with k % block_elems == 0: one warp per row, lanes
// over 32-value slabs, byte loads.  Correct everywhere, tuned nowhere; used
// for shapes the bulk path does not take.
template <int TYPE>
__device__ __forceinline__ float slab_dot(const uint8_t* __restrict__ row, int j, const uint8_t* __restrict__ xb) {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xb);
    const uint32_t ds = __ldg(xw);
    const float dx = half_lo(ds), sx = half_hi(ds);
    int q[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int word = static_cast<int>(__ldg(xw + 1 + i));
#pragma unroll
        for (int e = 0; e < 4; ++e) q[4 * i + e] = static_cast<int8_t>((word >> (8 * e)) & 255);
    }
    if (TYPE == P100_Q4_0) {
        const uint8_t* blk = row + size_t(j) * 18;
        const float d = load_half_bytes(blk);
        int dot = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) dot += (blk[2 + i] & 15) * q[i] + (blk[2 + i] >> 4) * q[i + 16];
        return d * fmaf(float(dot), dx, -8.0f * sx);
    } else if (TYPE == P100_Q8_0) {
        const uint8_t* blk = row + size_t(j) * 34;
        const float d = load_half_bytes(blk);
        int dot = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) dot += static_cast<int8_t>(blk[2 + i]) * q[i];
        return (d * dx) * float(dot);
    } else if (TYPE == P100_Q4_K || TYPE == P100_Q5_K) {
        constexpr int BB = TYPE == P100_Q4_K ? 144 : 176;
        const uint8_t* blk = row + size_t(j / 8) * BB;
        const int sub = j % 8;
        const float d = load_half_bytes(blk), dmin = load_half_bytes(blk + 2);
        int sc, mn;
        q4k_scale_min(blk + 4, sub, sc, mn);
        const uint8_t* qs = blk + (TYPE == P100_Q4_K ? 16 : 48) + (sub / 2) * 32;
        const uint8_t* qh = blk + 16;   // Q5_K: bit `sub` of qh[i] is the code's 16
        const int shift = (sub % 2) * 4;
        int dot = 0, sumq = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            int w = (qs[i] >> shift) & 15;
            if (TYPE == P100_Q5_K) w |= ((qh[i] >> sub) & 1) << 4;
            dot += w * q[i];
            sumq += q[i];
        }
        return fmaf(d, dx * float(dot * sc), -dmin * (dx * float(sumq * mn)));
    } else {
        // Q6_K: (d * dx) * (sc0 * dot(values 0..15) + sc1 * dot(values 16..31))
        const uint8_t* blk = row + size_t(j / 8) * 210;
        const int sub = j % 8, h = sub / 4, c = sub % 4;
        const float d = load_half_bytes(blk + 208);
        const uint8_t* ql = blk + 64 * h + 32 * (c & 1);
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + 2 * c);
        const int nshift = (c >> 1) * 4, hshift = 2 * c;
        int lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            lo += ((((ql[i] >> nshift) & 15) | (((qh[i] >> hshift) & 3) << 4)) - 32) * q[i];
            hi += ((((ql[i + 16] >> nshift) & 15) | (((qh[i + 16] >> hshift) & 3) << 4)) - 32) * q[i + 16];
        }
        return (d * dx) * float(sc[0] * lo + sc[1] * hi);
    }
}

template <int TYPE>
__global__ void __launch_bounds__(256) qmv_generic_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xq,
                                                          float* __restrict__ y, int rows, int k, int batch,
                                                          size_t row_bytes) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= rows) return;
    const int slabs = k / 32;
    const uint8_t* row = w + size_t(r) * row_bytes;
    for (int c = 0; c < batch; ++c) {
        float acc = 0.f;
        for (int j = lane; j < slabs; j += 32) acc += slab_dot<TYPE>(row, j, xq + (size_t(c) * slabs + j) * 36);
        acc = warp_sum(acc);
        if (lane == 0) y[size_t(c) * rows + r] = acc;
    }
}

}  // namespace qmv
}  // namespace p100b
