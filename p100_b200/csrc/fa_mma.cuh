// fa_mma.cuh — FlashAttention-vec decode with the dot products on the tensor
// cores (mma.sync m16n8k16, f16 inputs, f32 accumulation) at FP32-level
// accuracy.
//
// Decode attention is HBM-bound: the math is G query heads x D per key, and a
// SIMT kernel spends most of its instructions on shuffles, conversions and
// barriers around it.  Here each warp owns 16 keys of every 64-key tile and
// runs its own online softmax over them (no barrier inside a tile):
//   S = Q K^T   A = the query rows, B = K via ldmatrix from the stage;
//   O += P V    A = P straight from S's accumulator fragments (two 8-key
//               n-tiles make one 16-key k-step), B = V via ldmatrix.trans.
// Accuracy: the operands must be f16, so Q and P are split in two,
// x = hi + lo with hi = f16(x), lo = f16(x - hi): rows 0..G-1 of A carry hi,
// rows G..2G-1 carry lo, and the f32 accumulators add the halves back
// (K and V are f16 already, so S and O keep ~22 significant bits).  Q is
// scaled per head by a power of two so its largest entry sits near 2^13
// (no f16 overflow, lo well above the subnormals); S is scaled back exactly.
//
// K/V tiles are copied with 16-byte cp.async into rows padded to D + 8
// halves, so the eight 16-byte rows an ldmatrix reads fall on distinct banks;
// rows past the part's last key are zero-filled (a masked key's V then adds
// exactly 0).  The query is loaded into registers before the first K/V copy
// is issued (loads issued after 96 KB of copies waited ~2.6 us behind them).
// Split-K parts are those of fa_decode.cuh (fa::Params, partials {m, l,
// unnormalised O}); they are combined either by the last CTA through the
// global workspace, or, when the parts of a kv head form one thread-block
// cluster, through distributed shared memory: every CTA then merges its own
// slice of the outputs (no workspace, fence, ticket or L2 round trips).
//
// Quantised caches (KV = q8_0 or q4_0): the ring holds the raw blocks of
// each 64-key tile (the tile is one contiguous byte range of the head, copied
// in 16-byte chunks from the 16-byte boundary at or below its start), and
// each warp dequantises its own 16 rows of K and V into a private fp16 tile
// with the values of kvq::dequant8 (rows past the part's end as zeros), then
// runs the fp16 code on it unchanged — so the result is that of the fp16
// kernel on the converted cache, bit for bit, from about half (q8_0) or a
// quarter (q4_0) of the bytes.
#pragma once
#include "fa_decode.cuh"
#include "kv_quant.cuh"

namespace p100b {
namespace fam {

// Two shapes, chosen per call by the host: 4 warps over 64-key tiles (two
// or three CTAs per SM, the cluster merge up to 8K keys), or 8 warps over
// 128-key tiles (one CTA per SM with deeper rings, longer contexts: twice the
// warps per CTA hide the per-tile chain better than a second CTA does, and a
// split of one part per SM keeps the workspace merge short).  Each warp owns
// 16 keys of every tile.
template <int NW>
__host__ __device__ constexpr int tile_keys() { return 16 * NW; }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    return uint32_t(__half_as_ushort(__float2half_rn(lo))) | (uint32_t(__half_as_ushort(__float2half_rn(hi))) << 16);
}
// f16 residual of x: f16(x - f16(x))
__device__ __forceinline__ float half_rest(float x) { return x - __half2float(__float2half_rn(x)); }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// 8x8 b16 transpose within the warp: lane (g, t) gets elements (2t, g) and
// (2t+1, g) of the matrix whose (g, 2t..2t+1) it held.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
// Values i and i+1 (i even, within one block) of the block at byte offset
// `blk` of shared memory as an fp16 pair, rounded as kvq::dequant8 rounds.
template <int KV>
__device__ __forceinline__ uint32_t dequant_pair(const uint8_t* smem, int blk, int i, uint32_t d2) {
    uint32_t x;
    if (KV == P100_KV_Q8_0) {
        x = *reinterpret_cast<const unsigned short*>(smem + blk + 2 + i) ^ 0x8080u;
    } else {
        const uint32_t w = *reinterpret_cast<const unsigned short*>(smem + blk + 2 + (i & 15));
        x = (i < 16 ? w : w >> 4) & 0x0F0Fu;
    }
    uint32_t h = __byte_perm(x, 0x64u, 0x4140);
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(h) : "r"(KV == P100_KV_Q8_0 ? 0x64806480u : 0x64086408u));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h) : "r"(d2));
    return h;
}

// Every thread of the cluster arrives; release/acquire orders the shared
// memory written before it with the remote reads after it.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Stores v into CTA `rank`'s shared memory at the address of `local` in ours.
__device__ __forceinline__ void st_cluster(float* local, int rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Three stages: 64-key ones (107 KB of shared memory at D = 128) let two CTAs
// fit an SM, so a cluster of 16 parts per kv head fits a GPC (7 such clusters
// fit the GPU at four stages, 14 at three); 128-key ones take 218 KB.
template <int D>
__host__ __device__ constexpr int stages() { return D >= 256 ? 2 : 3; }
// Cluster-merge receive area: [16 parts][G][D] slices of O (G*D floats in
// all) and [16][G] m and l; its own region, so a peer that finishes early can
// store into it while this CTA still streams K/V.
constexpr int kMaxClusterParts = 16;
template <int D, int G>
__host__ __device__ constexpr size_t rx_floats() { return size_t(G) * D + 2 * kMaxClusterParts * G; }
// Quantised caches: bytes per key row, per raw K (or V) slot (the tile plus
// up to 15 bytes of lead before it, rounded up with room to spare), and as
// many stages (3 to 8) as leave three 4-warp CTAs per SM at G = 8 (76,800
// bytes per CTA), or fill one SM for the 8-warp shape (232,448 bytes).
template <int D, int KV>
__host__ __device__ constexpr int raw_row_bytes() { return D / 32 * kvq::block_bytes<KV>(); }
template <int D, int KV, int NW>
__host__ __device__ constexpr int raw_slot_bytes() { return (tile_keys<NW>() * raw_row_bytes<D, KV>() + 48 + 15) & ~15; }
constexpr int kQuantCtasPerSm = 3;   // 4-warp shape over a quantised cache
template <int NW>
__host__ __device__ constexpr int ctas_per_sm(int kv) { return NW == 8 ? 1 : kv == P100_KV_F16 ? 2 : kQuantCtasPerSm; }
template <int D, int NW>
__host__ __device__ constexpr int quant_ring_budget() {
    return (NW == 8 ? 232448 : 76800) - (8 * D * 4 + 256 + int(rx_floats<D, 8>()) * 4);
}
template <int D, int KV, int NW>
__host__ __device__ constexpr int nstages() {
    return KV == P100_KV_F16 ? stages<D>()
           : quant_ring_budget<D, NW>() / (2 * raw_slot_bytes<D, KV, NW>()) < 3 ? 3
           : quant_ring_budget<D, NW>() / (2 * raw_slot_bytes<D, KV, NW>()) > 8 ? 8
                                                                                : quant_ring_budget<D, NW>() / (2 * raw_slot_bytes<D, KV, NW>());
}
// fp16 stages hold [K|V][D/64 boxes][tile rows][128 B], 128-byte swizzled,
// from a 1024-byte boundary (the slack is the last 1024 bytes).
template <int D, int KV, int NW>
__host__ __device__ constexpr size_t ring_bytes() {
    return KV == P100_KV_F16 ? size_t(stages<D>()) * 2 * tile_keys<NW>() * D * 2 + 1024
                             : size_t(nstages<D, KV, NW>()) * 2 * raw_slot_bytes<D, KV, NW>();
}
template <int D, int G, int KV = P100_KV_F16, int NW = 4>
__host__ __device__ constexpr size_t smem_bytes() {
    return ring_bytes<D, KV, NW>() + size_t(G) * D * 4 + 256 + rx_floats<D, G>() * 4;
}
static_assert(smem_bytes<128, 8, P100_KV_Q8_0>() <= 76800 && smem_bytes<128, 8, P100_KV_Q4_0>() <= 76800 &&
                  smem_bytes<64, 8, P100_KV_Q8_0>() <= 76800 && smem_bytes<64, 8, P100_KV_Q4_0>() <= 76800,
              "three 4-warp CTAs per SM");
static_assert(smem_bytes<128, 8, P100_KV_F16, 8>() <= 232448 && smem_bytes<128, 8, P100_KV_Q8_0, 8>() <= 232448 &&
                  smem_bytes<128, 8, P100_KV_Q4_0, 8>() <= 232448,
              "one 8-warp CTA per SM");

// Grid (parts, batch * n_kv); G = query heads per kv head (1, 2, 4 or 8);
// D = 64 or 128; KV = the cache's p100_kv_type; NW = 4 or 8 warps.
template <int D, int G, int KV = P100_KV_F16, int NW = 4>
__global__ void __launch_bounds__(NW * 32, ctas_per_sm<NW>(KV)) fa_mma_kernel(const __grid_constant__ fa::Params p) {
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "G");
    static_assert(NW == 4 || NW == 8, "NW");
    constexpr int kWarps = NW, kThreads = NW * 32, kTile = tile_keys<NW>();
    constexpr int NS = nstages<D, KV, NW>();
    constexpr int KSQ = D / 16;      // k-steps of Q K^T
    constexpr int NTV = D / 8;       // n-tiles of P V
    constexpr bool QUANT = KV != P100_KV_F16;
    constexpr int BB = kvq::block_bytes<KV>();
    constexpr int RB = raw_row_bytes<D, KV>();
    constexpr int RAW = raw_slot_bytes<D, KV, NW>();
    extern __shared__ __align__(128) uint8_t smem[];
    // fp16: [NS][K|V][D/64][kTile][128 B] from the first 1024-byte boundary;
    // quantised: [NS][K|V][RAW] from the start
    uint8_t* ring = smem + (QUANT ? 0u : (1024u - (smem_addr(smem) & 1023u)) & 1023u);
    float* s_q = reinterpret_cast<float*>(smem + ring_bytes<D, KV, NW>());   // [G][D]
    float* s_qs = s_q + G * D;                                          // [8] per-head power-of-two scale
    unsigned* s_flag = reinterpret_cast<unsigned*>(s_qs + 8);
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_qs + 16);           // [NS] K/V stage barriers
    float* rx = reinterpret_cast<float*>(smem + smem_bytes<D, G, KV, NW>() - rx_floats<D, G>() * 4);   // cluster merge

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int bk = blockIdx.y, part = blockIdx.x;
    if (!QUANT && tid == 0) {   // the descriptors load while the query and barriers are set up
        prefetch_tensormap(&p.tmk);
        prefetch_tensormap(&p.tmv);
    }
    const int b = bk / p.nkv, kvh = bk % p.nkv;
    int seq = p.seq, pos = -1;
    if (p.rope_cs) {   // fused decode step: keys [0, pos], pos device-resident
        pdl_wait_prior_grid();
        pos = *p.len_dev;
        if (pos < 0 || pos >= p.seq) {
            if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicExch(&g_device_error, kDevErrInput);
            pos = -1;
        }
        seq = pos + 1;
    } else if (p.len_dev) {
        pdl_wait_prior_grid();
        seq = min(max(*p.len_dev + p.len_add, 0), p.seq);
    }
    const int key0 = static_cast<int>(static_cast<long long>(seq) * part / p.parts);
    const int key1 = static_cast<int>(static_cast<long long>(seq) * (part + 1) / p.parts);
    const int ntiles = (key1 - key0 + kTile - 1) / kTile;
    const __half* kbase = p.k + b * p.batch_stride + kvh * p.head_stride;
    const __half* vbase = p.v + b * p.batch_stride + kvh * p.head_stride;
    const uint32_t ring_addr = smem_addr(ring);
    // quantised: this head's rows (strides count values, in whole blocks)
    const size_t qhead = size_t((b * p.batch_stride + kvh * p.head_stride) / 32) * BB;
    const uint8_t* kq = reinterpret_cast<const uint8_t*>(p.k) + qhead;
    const uint8_t* vq = reinterpret_cast<const uint8_t*>(p.v) + qhead;
    // bytes before each tile's 16-byte boundary (the same for every tile: 64 rows are 256-byte multiples)
    const int lead_k = static_cast<int>(reinterpret_cast<uintptr_t>(kq + size_t(key0) * RB) & 15);
    const int lead_v = static_cast<int>(reinterpret_cast<uintptr_t>(vq + size_t(key0) * RB) & 15);

    // The raw query pairs of this group, loaded before any K/V copy is issued
    // (after the wait when they come from the previous kernel).
    constexpr int QPT = (G * D / 2 + kThreads - 1) / kThreads;   // pairs per thread
    const float* qg = p.q + (size_t(b) * p.nkv * G + size_t(kvh) * G) * D;
    float2 qr[QPT];
#pragma unroll
    for (int j = 0; j < QPT; ++j) {
        const int i = tid + j * kThreads;
        qr[j] = i < G * D / 2 ? *reinterpret_cast<const float2*>(qg + 2 * i) : make_float2(0.f, 0.f);
    }

    // fp16 K/V tiles: 16-byte cp.async chunks into rows padded to D + 8
    // halves (chunk i of this thread: row crow + i * RSTEP), zero-filled past
    // the part's end (a masked key's V then adds exactly 0); one commit group
    // per tile.  (Per-row bulk copies, 128 per tile, measured slower.)
    // Quantised tiles: the rows are one contiguous byte range of the head,
    // copied by one bulk-async copy from the 16-byte boundary `lead` bytes
    // below it, as far as 16-byte chunks stay inside the head's p.seq rows,
    // completing on the stage's mbarrier (thread 0 arms it); the rest (< 16
    // bytes, a multiple of 4) by plain 4-byte loads and stores, fenced
    // against the async proxy that refills the slot later and visible to
    // readers through the block barriers between issue and use.
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const uint64_t policy = l2_evict_first_policy();
    // quantised: the 16-byte aligned source of rows [j0, j0 + n), its whole
    // 16-byte chunks inside the head's rows, and the 4-byte words after them
    auto quant_part = [&](const uint8_t* head, int lead, int j0, int n, int& nfull, int& tail) {
        const uint8_t* src = head + size_t(j0) * RB - lead;
        const uintptr_t end = reinterpret_cast<uintptr_t>(head + size_t(p.seq) * RB);
        const int total = lead + n * RB;
        nfull = (total + 15) >> 4;
        if (reinterpret_cast<uintptr_t>(src) + size_t(nfull) * 16 > end)
            nfull = static_cast<int>(((end & ~uintptr_t(15)) - reinterpret_cast<uintptr_t>(src)) >> 4);
        tail = (total - nfull * 16) >> 2;
        return src;
    };
    auto issue = [&](int tile) {
        if (tile >= ntiles) return;
        const int j0 = key0 + tile * kTile;
        const int n = min(kTile, key1 - j0);
        uint64_t* bar = &bars[tile % NS];
        if constexpr (QUANT) {
            uint8_t* kdst = smem + (tile % NS) * 2 * RAW;
            uint8_t* vdst = kdst + RAW;
            int nk, tk, nv, tv;
            const uint8_t* ksrc = quant_part(kq, lead_k, j0, n, nk, tk);
            const uint8_t* vsrc = quant_part(vq, lead_v, j0, n, nv, tv);
            if (tid == 0) {
                mbar_arrive_expect_tx(bar, uint32_t(nk + nv) * 16);
                bulk_load(kdst, ksrc, uint32_t(nk) * 16, bar, policy);
                bulk_load(vdst, vsrc, uint32_t(nv) * 16, bar, policy);
            }
            if (tk > 0 || tv > 0) {   // the head's last rows only
                if (tid < tk)
                    *reinterpret_cast<uint32_t*>(kdst + nk * 16 + 4 * tid) =
                        *reinterpret_cast<const uint32_t*>(ksrc + nk * 16 + 4 * tid);
                if (tid >= 64 && tid - 64 < tv)
                    *reinterpret_cast<uint32_t*>(vdst + nv * 16 + 4 * (tid - 64)) =
                        *reinterpret_cast<const uint32_t*>(vsrc + nv * 16 + 4 * (tid - 64));
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
        } else if (tid == 0) {
            // D/64 boxes of 64 values x kTile rows each for K and V; rows past
            // the tensor's p.seq read as zeros, rows of the next part are
            // read and masked (their V rows are zeroed after the wait)
            (void)n;
            const uint32_t kdst = ring_addr + uint32_t((tile % NS) * 2 * kTile * D * 2);
            const uint32_t vdst = kdst + uint32_t(kTile * D * 2);
            mbar_arrive_expect_tx(bar, uint32_t(2 * kTile * D * 2));
#pragma unroll
            for (int bx = 0; bx < D / 64; ++bx) {
                tma_load_4d(kdst + uint32_t(bx * kTile * 128), &p.tmk, bx * 64, j0, kvh, b, bar, policy);
                tma_load_4d(vdst + uint32_t(bx * kTile * 128), &p.tmv, bx * 64, j0, kvh, b, bar, policy);
            }
        }
    };
    auto issue_tile = [&](int tile) { issue(tile); };

    if (!p.len_dev)
        for (int s = 0; s < NS - 1; ++s) issue_tile(s);   // K/V never come from the previous kernel here
    pdl_allow_dependents();
    pdl_wait_prior_grid();
    if (QUANT && p.rope_cs && pos >= 0 && part == p.parts - 1) {
        // the new row, quantised: warp w forms blocks w, w + 4, ... of the
        // rotated k row then of the v row (lane = value in the block; the
        // rotation pairs adjacent lanes) and stores them into row pos
        const float* kr = p.q + (size_t(p.nq_total) + kvh) * D;
        const float* vr = p.q + (size_t(p.nq_total) + p.nkv + kvh) * D;
        for (int blk = warp; blk < 2 * (D / 32); blk += kWarps) {
            const bool is_k = blk < D / 32;
            const int e = (is_k ? blk : blk - D / 32) * 32 + lane;
            float x;
            if (is_k) {
                const float xe = kr[e], xo = __shfl_xor_sync(0xffffffffu, xe, 1);
                const float x0 = (lane & 1) ? xo : xe, x1 = (lane & 1) ? xe : xo;
                const float2 t = p.rope_cs[size_t(pos) * (D / 2) + e / 2];
                x = (lane & 1) ? __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x))
                               : __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
            } else {
                x = vr[e];
            }
            uint8_t* row = const_cast<uint8_t*>(is_k ? kq : vq) + size_t(pos) * RB;
            kvq::quantize_block_warp<KV>(x, lane, row + (e / 32) * BB);
        }
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");   // the row is read by bulk copies next
        __syncthreads();
    } else if (p.rope_cs && pos >= 0 && part == p.parts - 1) {
        // the new row: rotated k and v of this kv head into cache row pos
        // (only this part's key range reaches pos), visible before any copy
        const float* kr = p.q + (size_t(p.nq_total) + kvh) * D;
        const float* vr = p.q + (size_t(p.nq_total) + p.nkv + kvh) * D;
        for (int i = tid; i < D / 2; i += kThreads) {
            const float2 t = p.rope_cs[size_t(pos) * (D / 2) + i];
            const float x0 = kr[2 * i], x1 = kr[2 * i + 1];
            const float y0 = __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
            const float y1 = __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x));
            *reinterpret_cast<__half2*>(const_cast<__half*>(kbase) + size_t(pos) * D + 2 * i) =
                __halves2half2(__float2half_rn(y0), __float2half_rn(y1));
            *reinterpret_cast<__half2*>(const_cast<__half*>(vbase) + size_t(pos) * D + 2 * i) =
                __halves2half2(__float2half_rn(vr[2 * i]), __float2half_rn(vr[2 * i + 1]));
        }
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");   // the row is read by bulk copies next
        __syncthreads();
    }
    if (p.len_dev)
        for (int s = 0; s < NS - 1; ++s) issue_tile(s);

    // ---- queries: q * scale per head, scaled by a power of two 2^e so the
    // largest |entry| lies in [2^13, 2^14)
    float2 qv2[QPT];   // this thread's pairs, rotated and scaled
#pragma unroll
    for (int j = 0; j < QPT; ++j) {
        const int i = tid + j * kThreads;
        if (i >= G * D / 2) break;
        const float x0 = qr[j].x, x1 = qr[j].y;
        if (p.rope_cs) {   // rotate the raw q pair (rope_kv_append_kernel's arithmetic)
            const int pr = pos >= 0 ? pos : 0;
            const float2 t = p.rope_cs[size_t(pr) * (D / 2) + i % (D / 2)];
            qv2[j] = make_float2(__fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y)) * p.scale,
                                 __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x)) * p.scale);
        } else {
            qv2[j] = make_float2(x0 * p.scale, x1 * p.scale);
        }
        s_q[2 * i] = qv2[j].x;
        s_q[2 * i + 1] = qv2[j].y;
    }
    __syncthreads();
    for (int h = warp; h < G; h += kWarps) {
        float m = 0.f;
        for (int d = lane; d < D; d += 32) m = fmaxf(m, fabsf(s_q[h * D + d]));
        m = warp_max(m);
        if (lane == 0) {
            // e = 13 - ilogb(m), clamped so 2^e and 2^-e stay normal floats;
            // from the exponent bits (a subnormal m clamps to 120 either way)
            int e = 0;
            if (m > 0.f && m < INFINITY) e = max(-120, min(120, 13 - (((__float_as_int(m) >> 23) & 255) - 127)));
            s_qs[h] = __int_as_float((e + 127) << 23);
        }
    }
    __syncthreads();
    // Each thread splits its own pairs x = q * 2^e into hi = fp16(x) and
    // lo = fp16(x - hi), over s_q (whose values were all read above): the A
    // fragments then load as fp16 pairs.
    __half2* s_hi = reinterpret_cast<__half2*>(s_q);   // [G * D / 2]
    __half2* s_lo = s_hi + G * D / 2;                   // [G * D / 2]
#pragma unroll
    for (int j = 0; j < QPT; ++j) {
        const int i = tid + j * kThreads;
        if (i >= G * D / 2) break;
        const float sc = s_qs[2 * i / D];
        const float x0 = qv2[j].x * sc, x1 = qv2[j].y * sc;
        const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
        s_hi[i] = __halves2half2(h0, h1);
        s_lo[i] = __halves2half2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
    }
    __syncthreads();
    // A fragments: row r < G -> hi of head r, G <= r < 2G -> lo of head r - G
    uint32_t qa[KSQ][4];
    {
        const uint32_t* hi32 = reinterpret_cast<const uint32_t*>(s_hi);
        const uint32_t* lo32 = reinterpret_cast<const uint32_t*>(s_lo);
        auto frag = [&](int r, int d) -> uint32_t {   // elements (r, d), (r, d + 1), d even
            if (r < G) return hi32[(r * D + d) / 2];
            if (r < 2 * G) return lo32[((r - G) * D + d) / 2];
            return 0u;
        };
#pragma unroll
        for (int ks = 0; ks < KSQ; ++ks) {
            const int d0 = ks * 16 + 2 * t;
            qa[ks][0] = frag(g, d0);
            qa[ks][1] = frag(g + 8, d0);
            qa[ks][2] = frag(g, d0 + 8);
            qa[ks][3] = frag(g + 8, d0 + 8);
        }
    }
    // this lane's head (rows g and, for G = 8, g + 8 belong to head g mod G)
    const int hh = g % G;
    const bool row_live = g < 2 * G;
    const float unscale = 1.0f / s_qs[hh];   // exact: a power of two

    float o[NTV][4];
#pragma unroll
    for (int n = 0; n < NTV; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    bool copies_ok = true;   // false once a stage wait gave up (device flag raised): stop waiting
    for (int tile = 0; tile < ntiles; ++tile) {
        const int j0 = key0 + tile * kTile;
        const int n = min(kTile, key1 - j0);
        // fp16: the stage's K and V boxes (128-byte swizzled: the 16-byte
        // chunk c of row r sits at chunk c ^ (r % 8))
        const uint32_t kst = ring_addr + uint32_t((tile % NS) * 2 * kTile * D * 2);
        const uint32_t vst = kst + uint32_t(kTile * D * 2);
        if (copies_ok) copies_ok = mbar_wait(&bars[tile % NS], (tile / NS) & 1);
        if (!QUANT && n < kTile) {
            // V rows past the part's end hold the next keys (or zeros past
            // the tensor): make them zeros so a masked key adds exactly 0
            for (int i = tid; i < (kTile - n) * (D / 8); i += kThreads) {
                const int r = n + i / (D / 8), c = i % (D / 8);
                *reinterpret_cast<uint4*>(ring + (vst - ring_addr) + (c >> 3) * kTile * 128 + r * 128 + (c & 7) * 16) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the slot is refilled by TMA later
        }
        __syncthreads();   // tile's copies visible to all; the slot refilled next is no longer read
        if (copies_ok) issue_tile(tile + NS - 1);
        // fp16: K and V fragments by ldmatrix from the stage.  Quantised:
        // straight from the raw rows — K pairs (key, dims 2t..2t+1) are the
        // B fragment as they stand, V pairs are transposed by movmatrix —
        // with the values kvq::dequant8 gives; V rows past n are zeros.
        const int kraw = (tile % NS) * 2 * RAW + lead_k, vraw = (tile % NS) * 2 * RAW + RAW + lead_v;
        auto scale2 = [&](int off) -> uint32_t {
            const uint32_t d = *reinterpret_cast<const unsigned short*>(smem + off);
            return d | (d << 16);
        };

        // ---- S = Q K^T over this warp's 16 keys (two n-tiles of 8)
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
            if constexpr (QUANT) {
                const int row = kraw + (warp * 16 + nt * 8 + g) * RB;
                uint32_t d2[D / 32];
#pragma unroll
                for (int bk = 0; bk < D / 32; ++bk) d2[bk] = scale2(row + bk * BB);
#pragma unroll
                for (int ks = 0; ks < KSQ; ++ks) {
                    const int j = ks * 16 + 2 * t;   // dims j, j+1 and j+8, j+9
                    const uint32_t b0 = dequant_pair<KV>(smem, row + (j / 32) * BB, j % 32, d2[j / 32]);
                    const uint32_t b1 = dequant_pair<KV>(smem, row + (j / 32) * BB, j % 32 + 8, d2[j / 32]);
                    mma16816(s[nt], qa[ks], b0, b1);
                }
            } else {
                const int krow = warp * 16 + nt * 8 + (lane & 7);
#pragma unroll
                for (int ks = 0; ks < KSQ; ks += 2) {
                    uint32_t r[4];
                    const int cidx = 2 * ks + (lane >> 3);   // 16-byte chunk of the row
                    ldsm_x4(r, kst + uint32_t((cidx >> 3) * kTile * 128 + krow * 128 + (((cidx & 7) ^ (krow & 7)) << 4)));
                    mma16816(s[nt], qa[ks], r[0], r[1]);
                    mma16816(s[nt], qa[ks + 1], r[2], r[3]);
                }
            }
        }
        // hi + lo rows -> the head's scores for keys (nt, 2t + e)
        float x[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float v;
                if (G == 8) {
                    v = s[nt][e] + s[nt][2 + e];
                } else {
                    v = s[nt][e] + __shfl_xor_sync(0xffffffffu, s[nt][e], 4 * G);
                }
                v *= unscale;
                if (p.softcap > 0.f) v = p.softcap * tanhf(v / p.softcap);
                const int kt = warp * 16 + nt * 8 + 2 * t + e;
                if (kt < n && p.mask) v += p.mask[j0 + kt];
                x[nt][e] = (kt < n && row_live) ? v : -INFINITY;
            }
        // ---- online softmax of this warp's keys, per head row
        float tmax = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        // m_new is shared by the four lanes of a row, but rows differ (unused
        // rows never see a key): the shuffles below run in every lane and only
        // rows with a visible key update m, l and O.
        const bool seen = m_new != -INFINITY;
        float alpha = 1.f, pr[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        if (seen) {
            alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) pr[nt][e] = expf(x[nt][e] - m_new);
        }
        float ps = (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        if (seen) {
            l_run = l_run * alpha + ps;
            m_run = m_new;
        }
        // ---- P as the A operand: rows < G hi, G..2G-1 lo (G = 8: row g+8 lo)
        uint32_t pa[4];
        if (G == 8) {
            pa[0] = pack_half2(pr[0][0], pr[0][1]);
            pa[1] = pack_half2(half_rest(pr[0][0]), half_rest(pr[0][1]));
            pa[2] = pack_half2(pr[1][0], pr[1][1]);
            pa[3] = pack_half2(half_rest(pr[1][0]), half_rest(pr[1][1]));
        } else {
            const bool lo = g >= G;
            pa[0] = !row_live ? 0u : lo ? pack_half2(half_rest(pr[0][0]), half_rest(pr[0][1]))
                                        : pack_half2(pr[0][0], pr[0][1]);
            pa[2] = !row_live ? 0u : lo ? pack_half2(half_rest(pr[1][0]), half_rest(pr[1][1]))
                                        : pack_half2(pr[1][0], pr[1][1]);
            pa[1] = pa[3] = 0u;
        }
        // ---- O = O * alpha + P V (no rows' maximum moved: alpha is 1 everywhere)
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
            for (int nv = 0; nv < NTV; ++nv) {
                o[nv][0] *= alpha;
                o[nv][1] *= alpha;
                o[nv][2] *= alpha;
                o[nv][3] *= alpha;
            }
        }
        if constexpr (QUANT) {
            // rows g and g + 8 of this warp's 16 keys; pairs (key, dims) -> (dims, key)
            const int r0 = warp * 16 + g;
            const bool ok0 = r0 < n, ok1 = r0 + 8 < n;
            const int row0 = vraw + r0 * RB, row1 = row0 + 8 * RB;
            uint32_t d0[D / 32], d1[D / 32];
#pragma unroll
            for (int bk = 0; bk < D / 32; ++bk) {
                d0[bk] = scale2(row0 + bk * BB);
                d1[bk] = scale2(row1 + bk * BB);
            }
            if (n == kTile) {
#pragma unroll
                for (int nv = 0; nv < NTV; ++nv) {
                    const int j = nv * 8 + 2 * t, bk = j / 32;
                    const uint32_t h0 = dequant_pair<KV>(smem, row0 + bk * BB, j % 32, d0[bk]);
                    const uint32_t h1 = dequant_pair<KV>(smem, row1 + bk * BB, j % 32, d1[bk]);
                    mma16816(o[nv], pa, movmatrix_trans(h0), movmatrix_trans(h1));
                }
            } else {
#pragma unroll
                for (int nv = 0; nv < NTV; ++nv) {
                    const int j = nv * 8 + 2 * t, bk = j / 32;
                    const uint32_t h0 = dequant_pair<KV>(smem, row0 + bk * BB, j % 32, d0[bk]);
                    const uint32_t h1 = dequant_pair<KV>(smem, row1 + bk * BB, j % 32, d1[bk]);
                    mma16816(o[nv], pa, movmatrix_trans(ok0 ? h0 : 0u), movmatrix_trans(ok1 ? h1 : 0u));
                }
            }
        } else {
#pragma unroll
            for (int n2 = 0; n2 < NTV / 2; ++n2) {
                uint32_t r[4];
                const int m = lane >> 3;
                const int vrow = warp * 16 + (lane & 7) + 8 * (m & 1);
                const int cidx = 2 * n2 + (m >> 1);
                ldsm_x4_trans(r, vst + uint32_t((cidx >> 3) * kTile * 128 + vrow * 128 + (((cidx & 7) ^ (vrow & 7)) << 4)));
                mma16816(o[2 * n2], pa, r[0], r[1]);
                mma16816(o[2 * n2 + 1], pa, r[2], r[3]);
            }
        }
    }
    __syncthreads();   // every copy landed (each issued tile was waited for) and every warp is done with the ring

    // ---- hi + lo rows of O; then merge the four warps through shared memory
    float* s_wm = reinterpret_cast<float*>(smem);          // [kWarps][8]
    float* s_wl = s_wm + kWarps * 8;                        // [kWarps][8]
    float* s_wo = s_wl + kWarps * 8;                        // [kWarps][G][D]
#pragma unroll
    for (int nv = 0; nv < NTV; ++nv)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float v;
            if (G == 8) {
                v = o[nv][e] + o[nv][2 + e];
            } else {
                v = o[nv][e] + __shfl_xor_sync(0xffffffffu, o[nv][e], 4 * G);
            }
            if (g < G) s_wo[(warp * G + g) * D + nv * 8 + 2 * t + e] = v;
        }
    if (g < G && t == 0) {
        s_wm[warp * 8 + g] = m_run;
        s_wl[warp * 8 + g] = l_run;
    }
    __syncthreads();
    float* s_m = s_wo + kWarps * G * D;   // [G]
    float* s_l = s_m + 8;                 // [G]
    float* s_ww = s_l + 8;                // [kWarps][8] rebase weights exp(m_w - m)
    if (tid < G) {
        float m = -INFINITY;
        for (int w = 0; w < kWarps; ++w) m = fmaxf(m, s_wm[w * 8 + tid]);
        float l = 0.f;
        for (int w = 0; w < kWarps; ++w) {
            const float lw = s_wl[w * 8 + tid];
            const float wt = lw != 0.f ? expf(s_wm[w * 8 + tid] - m) : 0.f;
            s_ww[w * 8 + tid] = wt;
            if (lw != 0.f) l = fmaf(wt, lw, l);
        }
        s_m[tid] = m;
        s_l[tid] = l;
    }
    __syncthreads();
    float* red = s_ww + kWarps * 8;   // [G][D] the CTA's unnormalised O
    for (int i = tid; i < G * D; i += kThreads) {
        const int h = i / D;
        float acc = 0.f;
        for (int w = 0; w < kWarps; ++w)
            if (s_wl[w * 8 + h] != 0.f) acc = fmaf(s_ww[w * 8 + h], s_wo[(w * G + h) * D + (i % D)], acc);
        red[i] = acc;
    }
    __syncthreads();

    const size_t row0 = size_t(b) * p.nkv * G + size_t(kvh) * G;   // first query head row
    if (p.cluster_merge) {
        // The parts of this kv head are the CTAs of one cluster (rank =
        // part); CTA q owns outputs [q*per, (q+1)*per) of the G x D block.
        // Every CTA stores its m, l (to all) and each owner's slice of its
        // unnormalised O into the owners' receive areas, one cluster barrier
        // makes them visible, and each CTA merges its slice from its own
        // shared memory with merge_parts' arithmetic, parts in order.  After
        // the barrier no CTA touches another's memory, so no second barrier.
        const int np = p.parts, per = G * D / np;
        float* rx_o = rx;                 // [np][per]
        float* rx_m = rx + G * D;         // [np][G]
        float* rx_l = rx_m + np * G;      // [np][G]
        for (int i = tid; i < G * D; i += kThreads) st_cluster(rx_o + part * per + i % per, i / per, red[i]);
        for (int i = tid; i < np * G; i += kThreads) {
            const int q = i / G, h = i % G;
            st_cluster(rx_m + part * G + h, q, s_m[h]);
            st_cluster(rx_l + part * G + h, q, s_l[h]);
        }
        cluster_barrier();
        float* s_w = red + G * D;         // [np][G] weights (local scratch)
        float* s_gm = s_w + np * G;       // [G]
        float* s_den = s_gm + G;          // [G]
        float* s_out = s_den + G;         // [per] this CTA's merged outputs
        // one warp per head, one lane per part (np <= 16): the global max,
        // the parts' weights exp(m_q - M) and den = sum of weight * l_q
        for (int h = warp; h < G; h += kWarps) {
            const bool has = lane < np;
            const float mq = has ? rx_m[lane * G + h] : -INFINITY;
            const float lq = has ? rx_l[lane * G + h] : 0.f;
            const float gmax = warp_max(mq);
            const float wq = lq == 0.f ? 0.f : expf(mq - gmax);
            const float den = warp_sum(wq * lq);
            if (has) s_w[lane * G + h] = wq;
            if (lane == 0) {
                s_gm[h] = gmax;
                s_den[h] = den;
                if (part == 0 && p.lse) p.lse[row0 + h] = den == 0.f ? -INFINITY : gmax + logf(den);
            }
        }
        __syncthreads();
        for (int i = tid; i < per; i += kThreads) {
            const int idx = part * per + i, h = idx / D;
            float num = 0.f;
#pragma unroll 8
            for (int q = 0; q < np; ++q)
                if (rx_l[q * G + h] != 0.f) num = fmaf(s_w[q * G + h], rx_o[q * per + i], num);
            const float den = s_den[h];
            const float o = den == 0.f ? 0.f : num / den;
            p.o[(row0 + h) * D + (idx % D)] = o;
            s_out[i] = o;
        }
        if (p.o_q81) {   // per is a multiple of 32: whole Q8_1 blocks
            __syncthreads();
            for (int j = warp; j < per / 32; j += kWarps)
                warp_q8_1_block(s_out[j * 32 + lane], lane, p.o_q81 + (row0 * D / 32 + part * per / 32 + j) * 36);
        }
        return;
    }
    if (p.parts == 1) {
        for (int i = tid; i < G * D; i += kThreads) {
            const int h = i / D, d = i % D;
            const float l = s_l[h];
            const float o = l == 0.f ? 0.f : red[i] / l;
            p.o[(row0 + h) * D + d] = o;
            red[i] = o;
            if (d == 0 && p.lse) p.lse[row0 + h] = l == 0.f ? -INFINITY : s_m[h] + logf(l);
        }
        if (p.o_q81) {
            __syncthreads();
            for (int j = warp; j < G * D / 32; j += kWarps)
                warp_q8_1_block(red[j * 32 + lane], lane, p.o_q81 + (row0 * D / 32 + j) * 36);
        }
        return;
    }
    float* my_o = p.ws_o + (size_t(bk) * p.parts + part) * G * D;
    float* my_ml = p.ws_ml + (size_t(bk) * p.parts + part) * G * 2;
    for (int i = tid; i < G * D; i += kThreads) my_o[i] = red[i];
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

    // Last CTA of this kv head: merge the parts (scratch past the CTA's own
    // partial sums in shared memory).
    fa::merge_parts<kThreads>(p, bk, G, D, row0, red + G * D);
}

}  // namespace fam
}  // namespace p100b
