// qmv.cuh — quantised mat-vec y = W x for Q4_0 / Q8_0 / Q4_K weights against
// Q8_1 activations, batch 1..16, on CUDA cores (int8 dp4a).
//
// Bulk path (16-byte aligned rows, k % 256 == 0):
//   * Each CTA owns a contiguous, balanced range of rows.  Its weight bytes are
//     one contiguous span of the matrix, streamed HBM -> shared memory in
//     stages of whole rows by untiled bulk-async copies (cp.async.bulk, L2
//     evict-first) into a ring of up to 4 stages with one mbarrier each.
//   * A row is cut into "items" of 64 weights: two Q4_0 or Q8_0 blocks, or a
//     quarter Q4_K super-block (its 16-byte header plus 32 bytes of nibbles).
//     Thread (group g, index t) always owns items t, t+T' of every row, so its
//     Q8_1 activations for those items are loaded once into registers; the
//     groups split each stage's rows.
//   * Per row, a warp sums its items' products with an XOR butterfly and
//     lane 0 writes one partial; after the stage barrier the partials of a row
//     are added in warp order.  The output is deterministic.
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

constexpr int kThreads = 256;
constexpr int kMaxStages = 4;
constexpr int kStageCap = 32 * 1024;      // target bytes per stage
constexpr int kSmemLimit = 227 * 1024;

// Activation operands of one item (two 32-value blocks) for one column.
struct ItemAct {
    int q[16];     // int8 codes of blocks 2*it and 2*it+1, four per word
    float f[4];    // Q4_0: dxA, sumA, dxB, sumB; Q8_0: dxA, dxB; Q4_K: dx0, dx1, sumq0, sumq1
};

struct Params {
    const uint8_t* w;
    const uint8_t* xq;     // block_q8_1 rows, 36 bytes per 32 values
    float* y;
    int rows, k;
    int col0;              // first activation column of this launch
    int row_bytes;
    int ipr;               // items per row = k / 64
    int tpr;               // threads per row group (multiple of 32)
    int groups;            // row groups per CTA
    int rps;               // rows per stage (multiple of groups)
    int nstage;
    int slot_bytes;        // ring slot stride (multiple of 128)
    int part_floats;       // floats per partial buffer
};

__device__ __forceinline__ void load_item_act(int type, const uint8_t* __restrict__ xq, int nb, int col, int it,
                                              ItemAct& a) {
    const uint32_t* blk = reinterpret_cast<const uint32_t*>(xq + (size_t(col) * nb + 2 * it) * 36);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t ds = __ldg(blk + 9 * h);
        int sumq = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            a.q[8 * h + i] = static_cast<int>(__ldg(blk + 9 * h + 1 + i));
            sumq = __dp4a(a.q[8 * h + i], 0x01010101, sumq);
        }
        if (type == P100_Q4_0) {
            a.f[2 * h] = half_lo(ds);
            a.f[2 * h + 1] = half_hi(ds);
        } else if (type == P100_Q8_0) {
            a.f[h] = half_lo(ds);
        } else {
            a.f[h] = half_lo(ds);
            a.f[2 + h] = float(sumq);
        }
    }
}

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
            int sa = 0, sb = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // byte m: low nibble is element m, high nibble element m+16
                sa = __dp4a(static_cast<int>(qa[i] & 0x0f0f0f0fu), a[c].q[i], sa);
                sa = __dp4a(static_cast<int>((qa[i] >> 4) & 0x0f0f0f0fu), a[c].q[4 + i], sa);
                sb = __dp4a(static_cast<int>(qb[i] & 0x0f0f0f0fu), a[c].q[8 + i], sb);
                sb = __dp4a(static_cast<int>((qb[i] >> 4) & 0x0f0f0f0fu), a[c].q[12 + i], sb);
            }
            // d_w * (d_x * sum(nib*q) - 8 * sum(x)): the -8 offset through the
            // block sum, as the q81 path does per half block.
            acc[c] = fmaf(dA, fmaf(float(sa), a[c].f[0], -8.0f * a[c].f[1]), acc[c]);
            acc[c] = fmaf(dB, fmaf(float(sb), a[c].f[2], -8.0f * a[c].f[3]), acc[c]);
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
            int sa = 0, sb = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                sa = __dp4a(qa[i], a[c].q[i], sa);
                sb = __dp4a(static_cast<int>(W[9 + i]), a[c].q[8 + i], sb);
            }
            acc[c] = fmaf(dA * a[c].f[0], float(sa), acc[c]);
            acc[c] = fmaf(dB * a[c].f[1], float(sb), acc[c]);
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
            int s0 = 0, s1 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                s0 = __dp4a(static_cast<int>(N[i] & 0x0f0f0f0fu), a[c].q[i], s0);
                s1 = __dp4a(static_cast<int>((N[i] >> 4) & 0x0f0f0f0fu), a[c].q[8 + i], s1);
            }
            // d * sum_j dx_j*(dot_j*sc_j) - dmin * sum_j dx_j*(sumq_j*mn_j)
            // (qmv_model.cpp:175-178, summed over both sub-blocks)
            const float sd = fmaf(a[c].f[0], float(s0 * sc0), a[c].f[1] * float(s1 * sc1));
            const float sm = fmaf(a[c].f[0], a[c].f[2] * float(mn0), a[c].f[1] * (a[c].f[3] * float(mn1)));
            acc[c] = fmaf(d, sd, acc[c]);
            acc[c] = fmaf(-dmin, sm, acc[c]);
        }
    }
}

template <int TYPE, int B, int IPT>
__global__ void __launch_bounds__(kThreads, 1) qmv_bulk_kernel(const Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);                    // kMaxStages barriers
    float* partial = reinterpret_cast<float*>(smem + 128);                // 2 buffers
    uint8_t* ring = smem + 128 + ((2 * p.part_floats * 4 + 127) & ~127);

    const int tid = threadIdx.x, lane = tid & 31;
    const int g = tid / p.tpr, t = tid % p.tpr;
    const bool active = g < p.groups;
    const int wpg = p.tpr >> 5;                 // warps per row group
    const int wig = t >> 5;                     // warp index within the group

    const int r0 = static_cast<int>(static_cast<long long>(p.rows) * blockIdx.x / gridDim.x);
    const int r1 = static_cast<int>(static_cast<long long>(p.rows) * (blockIdx.x + 1) / gridDim.x);
    const int nst = (r1 - r0 + p.rps - 1) / p.rps;

    if (tid == 0) {
        for (int s = 0; s < p.nstage; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();

    uint64_t policy = 0;
    auto issue = [&](int s) {
        const int slot = s % p.nstage;
        const int first = r0 + s * p.rps;
        const int nr = min(p.rps, r1 - first);
        const uint32_t bytes = static_cast<uint32_t>(nr) * p.row_bytes;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_load(ring + size_t(slot) * p.slot_bytes, p.w + size_t(first) * p.row_bytes, bytes, &full[slot], policy);
    };
    if (tid == 0) {
        policy = l2_evict_first_policy();
        for (int s = 0; s < min(p.nstage, nst); ++s) issue(s);
    }
    // Weights never depend on the previous kernel; activations may.
    pdl_allow_dependents();
    pdl_wait_prior_grid();

    const int nb = p.k / 32;
    ItemAct act[IPT][B];
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        const int it = t + u * p.tpr;
#pragma unroll
        for (int c = 0; c < B; ++c) {
            if (active && it < p.ipr) {
                load_item_act(TYPE, p.xq, nb, p.col0 + c, it, act[u][c]);
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) act[u][c].q[i] = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) act[u][c].f[i] = 0.f;
            }
        }
    }

    bool ok = true;
    for (int s = 0; s < nst; ++s) {
        const int slot = s % p.nstage;
        const bool timed_out = !mbar_wait(&full[slot], (s / p.nstage) & 1);
        const uint8_t* stage = ring + size_t(slot) * p.slot_bytes;
        const int first = r0 + s * p.rps;
        const int nr = min(p.rps, r1 - first);
        float* part = partial + (s & 1) * p.part_floats;
        if (active) {
            for (int rl = g; rl < nr; rl += p.groups) {
                const uint8_t* row = stage + size_t(rl) * p.row_bytes;
                float acc[B];
#pragma unroll
                for (int c = 0; c < B; ++c) acc[c] = 0.f;
#pragma unroll
                for (int u = 0; u < IPT; ++u) {
                    const int it = t + u * p.tpr;
                    if (it < p.ipr) {
                        float tmp[B];
#pragma unroll
                        for (int c = 0; c < B; ++c) tmp[c] = 0.f;
                        item_dot<TYPE, B>(row, it, act[u], tmp);
#pragma unroll
                        for (int c = 0; c < B; ++c) acc[c] += tmp[c];
                    }
                }
#pragma unroll
                for (int c = 0; c < B; ++c) {
                    const float v = warp_sum(acc[c]);
                    if (lane == 0) part[(c * p.rps + rl) * wpg + wig] = v;
                }
            }
        }
        // Slot fully read and this stage's partials visible.  A timed-out wait
        // is decided for the whole CTA here, so every thread leaves together.
        if (__syncthreads_or(timed_out)) {
            ok = false;
            break;
        }
        if (tid == 0 && s + p.nstage < nst) issue(s + p.nstage);
        if (tid < nr * B) {
            const int c = tid / nr, rl = tid % nr;
            float v = 0.f;
            for (int w = 0; w < wpg; ++w) v += part[(c * p.rps + rl) * wpg + w];
            p.y[size_t(p.col0 + c) * p.rows + first + rl] = v;
        }
    }
    if (!ok) {
        // Drain this CTA's own copies (bounded) before its shared memory goes away.
        if (tid == 0)
            for (int s = 0; s < min(p.nstage, nst); ++s) (void)mbar_wait(&full[s], 0);
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
    } else {
        const uint8_t* blk = row + size_t(j / 8) * 144;
        const int sub = j % 8;
        const float d = load_half_bytes(blk), dmin = load_half_bytes(blk + 2);
        int sc, mn;
        q4k_scale_min(blk + 4, sub, sc, mn);
        const uint8_t* qs = blk + 16 + (sub / 2) * 32;
        const int shift = (sub % 2) * 4;
        int dot = 0, sumq = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            dot += ((qs[i] >> shift) & 15) * q[i];
            sumq += q[i];
        }
        return fmaf(d, dx * float(dot * sc), -dmin * (dx * float(sumq * mn)));
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
