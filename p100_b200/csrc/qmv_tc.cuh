// qmv_tc.cuh — batched quantised mat-vec (batch 2..16) on the 5th-generation
// tensor cores: tcgen05.mma kind::i8, operand A and the accumulators in
// tensor memory.
//
// y[c][row] = sum over 32-value blocks b of the q81 block formula of
// qmv_model.cpp:147-180: an exact int32 dot of the block's weight codes with
// the column's Q8_1 codes, then the block's FP32 scaling.  The integer dots
// are what the tensor cores compute; the scaling differs per block (weight
// scale per row and block, activation scale and sum per column and block),
// so every block gets an accumulator of its own: one MMA of M = 128 rows, N
// = 16 columns, K = 32 (exactly one block) adds the block's 128 x 16 int32
// dots into a tensor-memory tile that holds the bits of 1.5 * 2^23, so the
// epilogue reads 1.5 * 2^23 + dot as a float (exact for |dot| < 2^22; a
// block's dot is below 2^19) and one packed f32x2 subtraction gives float(dot)
// for two columns, with no int-to-float conversion.  The epilogue writes the
// bias back into the tile after reading it and applies the block's scales
// while it adds the dots into FP32 sums held in registers (a thread per row).
//
// One CTA = 128 rows x (a K slice) x 16 columns; long rows are split over a
// cluster of up to 8 CTAs along K, whose row sums are added in slice order
// through distributed shared memory.  Warp roles (448 threads):
//   warp 12     producer: TMA tensor loads of raw weight stages (128 rows x
//               one 256-value group per row, the GGUF bytes unmodified) and of
//               the stage's activation blocks (the batch's columns) into a
//               ring of raw slots;
//   warps 0-3   converters (thread = row = tensor-memory lane): the row's
//               group read as 16-byte words, every block cut out in registers
//               (Q4_0 / Q4_K low nibbles are a block's first 16 values, high
//               nibbles the next 16) and stored into tensor memory as the
//               stage's A operands with one tcgen05.st; the weight scales of
//               the stage into shared memory; the batch's activation blocks
//               into B tiles (UMMA canonical K-major layout, no swizzle) and
//               activation scales;
//   warp 13     MMA issuer (one lane): 8 MMAs a stage, A from tensor memory,
//               B from shared memory, tcgen05.commit onto the stage's
//               mbarrier; this warp also allocates and frees tensor memory;
//   warps 4-11  epilogue, two warpgroups (thread = row = tensor-memory lane),
//               each taking four of a stage's blocks: tcgen05.ld of the
//               columns the batch uses, the bias written back, each block's
//               scaling in packed f32x2 arithmetic; the two warpgroups' sums
//               are added at the end in a fixed order.
// Operands are four stages deep (A in tensor memory, B tiles and scales in
// shared memory), freed together when the epilogue is done with a stage, so
// the converters run up to four stages ahead of it; the accumulators are two
// stages deep.
//
// Every wait is bounded (kWaitLimitNs); a role that gives up raises the
// device flag and the CTA's abort word, the others see it and leave, and the
// allocating warp frees tensor memory after the whole CTA has met.
#pragma once
#include <cudaTypedefs.h>

#include "common.cuh"
#include "qmv_mma.cuh"

namespace p100b {
namespace qmvtc {

constexpr int kRows = 128;            // M: rows per CTA (tensor-memory lanes)
constexpr int kCols = 16;             // N: activation columns (batch <= 16, zero-padded)
constexpr int kBlocks = 8;            // 32-value blocks per stage (one 256-value group)
constexpr int kTmemStages = 2;        // accumulator stages in tensor memory
constexpr int kOpSlots = 4;           // operand stages: A in tensor memory, B tiles and scales in shared memory
constexpr int kTmemCols = 512;        // the allocation (a power of two)
constexpr int kACol = kTmemStages * kBlocks * kCols;   // 256: A operands after the accumulators
constexpr int kAColsPerStage = kBlocks * 8;           // 32 int8 values of 128 rows = 8 columns a block
constexpr int kConvWarps = 4, kEpiWarps = 8;
constexpr int kThreads = (kConvWarps + kEpiWarps + 2) * 32;   // + producer warp + MMA warp
constexpr int kProducerWarp = 12, kMmaWarp = 13;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kMaxRaw = 8;            // raw stages in the ring at most
constexpr int kActRow = kBlocks * 36;            // one column's Q8_1 blocks of a stage: 288 B
constexpr int kActBytes = kCols * kActRow;       // activation slot: 4608 B
constexpr uint32_t kBias = 0x4B400000u;          // the bits of 1.5 * 2^23

static_assert(kACol + kOpSlots * kAColsPerStage <= kTmemCols, "tensor memory layout");

// Per shared-memory operand slot: B tiles [kBlocks][512 B], then FP32
// scales: weight [kBlocks][2][kRows] (scale and, for Q4_K, min term),
// activation [kBlocks][2][kCols] (d; -8 sum for Q4_0 / code sum for Q4_K).
constexpr int kBTile = kCols * 32;                         // 512 B
constexpr int kOpB = 0;
constexpr int kOpWs = kOpB + kBlocks * kBTile;             // 4096
constexpr int kOpXs = kOpWs + kBlocks * 2 * kRows * 4;     // + 8192
constexpr int kOpBytes = kOpXs + kBlocks * 2 * kCols * 4;  // + 1024 = 13312

struct Params {
    const uint8_t* xq;   // batch x k/32 Q8_1 blocks of 36 bytes, column-major
    float* y;            // [batch][rows]
    int rows, k, batch;
    int slices;          // K split over a cluster of this many CTAs
    int raw_slots;       // raw weight stages in the ring
    int raw_bytes;       // one raw stage's weights: kRows x group bytes
    int group_bytes;     // bytes of one 256-value group of a row
    CUtensorMap tmw;     // the weights as [rows][row_bytes / 2] uint16 units, box (group/2, kRows)
    CUtensorMap tmx;     // the Q8_1 rows as [batch][k/32*36 / 2] uint16 units, box (144, batch)
};

// ------------------------------------------------------------ tcgen05 wrappers
// Shared-memory matrix descriptor (sm_100): start address, leading and
// stride byte offsets in 16-byte units, descriptor version 1, no swizzle.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3fffu);
    d |= uint64_t((lbo >> 4) & 0x3fffu) << 16;
    d |= uint64_t((sbo >> 4) & 0x3fffu) << 32;
    d |= uint64_t(1) << 46;   // version
    return d;                 // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::i8: int32 accumulate, A and B K-major,
// N = 16, M = 128; a_signed / b_signed select s8 or u8.
__host__ __device__ constexpr uint32_t idesc_i8(bool a_signed, bool b_signed) {
    return (2u << 4)                          // D format: s32
           | (uint32_t(a_signed) << 7)        // A: 0 u8, 1 s8
           | (uint32_t(b_signed) << 10)       // B
           | (uint32_t(kCols >> 3) << 17)     // N >> 3
           | (uint32_t(kRows >> 4) << 24);    // M >> 4
}

// D (tensor memory) += A (tensor memory) * B (shared memory), int32.
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(1u)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// N consecutive 32-bit columns of this warp's 32 tensor-memory lanes (the
// 32x32b shape: thread i of the warp holds lane i), N in {4, 8, 16, 64}.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
    static_assert(N == 4 || N == 8 || N == 16 || N == 64, "tcgen05.ld width");
    if constexpr (N == 4)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
            : "r"(taddr)
            : "memory");
    if constexpr (N == 8)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
            : "r"(taddr)
            : "memory");
    if constexpr (N == 16)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
            "%13, %14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
              "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr)
            : "memory");
    if constexpr (N == 64)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
            "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
            "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, "
            "%51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
              "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
              "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
              "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
              "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
              "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
              "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
              "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
            : "r"(taddr)
            : "memory");
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&r)[N]) {
    static_assert(N == 64, "tcgen05.st width");
    if constexpr (N == 64)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
            "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
            "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, "
            "%51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};"
            :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
               "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
               "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
               "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]),
               "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]),
               "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]),
               "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]),
               "r"(r[63])
            : "memory");
}
// The same word into N consecutive columns of this warp's lanes.
template <int N>
__device__ __forceinline__ void tmem_fill(uint32_t taddr, uint32_t v) {
    static_assert(N == 4 || N == 8 || N == 16 || N == 64, "tcgen05.st width");
    if constexpr (N == 4)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};"
            ::"r"(taddr), "r"(v)
            : "memory");
    if constexpr (N == 8)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};"
            ::"r"(taddr), "r"(v)
            : "memory");
    if constexpr (N == 16)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
            "%1, %1, %1};"
            ::"r"(taddr), "r"(v)
            : "memory");
    if constexpr (N == 64)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
            "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
            "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
            "%1, %1, %1};"
            ::"r"(taddr), "r"(v)
            : "memory");
}

// 2-d tiled TMA load of box (c0, c1) of the map into dst, completing on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Bounded mbarrier wait that also ends when the CTA's abort word is set.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_word) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort_word) return false;
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicExch(&g_device_error, kDevErrTimeout);
            *abort_word = 1;
            return false;
        }
    }
}

// ------------------------------------------------------------ converters
// Bytes of one 256-value group of a row: eight Q4_0 / Q8_0 blocks or one
// Q4_K super-block.
template <int TYPE>
__host__ __device__ constexpr int group_bytes_of() {
    return TYPE == P100_Q8_0 ? 272 : 144;
}

// Byte offset of (column i, 16-byte chunk c) in a canonical K-major B tile:
// 8-column core matrices of 128 bytes, the two K chunks 128 bytes apart,
// 8-column groups 256 bytes apart (LBO 128, SBO 256).
__device__ __forceinline__ uint32_t canon(int i, int c) { return uint32_t((i >> 3) * 256 + c * 128 + (i & 7) * 16); }

// Row t's group of one stage (raw: kRows rows of group_bytes_of<TYPE>()) into
// its 64 A words in tensor memory (block j in columns 8 j .. 8 j + 7, the
// block's 32 codes in K order, four to a column) and the row's weight scales
// (ws: [kBlocks][2][kRows]).  t is this thread's tensor-memory lane.
template <int TYPE>
__device__ __forceinline__ void convert_weights(const uint8_t* raw, float* ws, uint32_t tmem_a, int t) {
    // the row as 16-byte loads (rows are 144 or 272 bytes apart, so eight
    // consecutive rows hit eight different 16-byte bank groups)
    constexpr int kWords = group_bytes_of<TYPE>() / 4;
    uint32_t w[kWords];
    const uint4* src = reinterpret_cast<const uint4*>(raw + size_t(t) * group_bytes_of<TYPE>());
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i) {
        const uint4 v = src[i];
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
    }
    uint32_t a[kAColsPerStage];
    constexpr uint32_t kLo = 0x0f0f0f0fu;
    if constexpr (TYPE == P100_Q4_0 || TYPE == P100_Q8_0) {
        constexpr int kB = TYPE == P100_Q4_0 ? 18 : 34;   // block bytes: fp16 d, then the codes
        constexpr int kN = TYPE == P100_Q4_0 ? 4 : 8;     // code words
#pragma unroll
        for (int j = 0; j < kBlocks; ++j) {
            const int b = kB * j;   // compile-time after unrolling
            uint32_t q[kN];
            float d;
            if ((b & 3) == 0) {   // d in the low half of a word, the codes 2 bytes into it
                d = half_lo(w[b / 4]);
#pragma unroll
                for (int i = 0; i < kN; ++i) q[i] = shift2(w[b / 4 + i], w[b / 4 + i + 1]);
            } else {              // d in the high half, the codes word-aligned after it
                d = half_hi(w[b / 4]);
#pragma unroll
                for (int i = 0; i < kN; ++i) q[i] = w[b / 4 + 1 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if constexpr (TYPE == P100_Q4_0)
                    a[8 * j + i] = i < 4 ? (q[i] & kLo) : ((q[i - 4] >> 4) & kLo);
                else
                    a[8 * j + i] = q[i];
            }
            ws[(j * 2) * kRows + t] = d;
        }
    } else {   // Q4_K: d, dmin | scales[12] | qs[128]; sub-block j = nibble half (j & 1) of qs bytes 32 (j / 2) ..
        const float d = half_lo(w[0]), dmin = half_hi(w[0]);
        auto sc = [&](int i) { return int((w[1 + i / 4] >> (8 * (i % 4))) & 255u); };
#pragma unroll
        for (int j = 0; j < kBlocks; ++j) {
            // get_scale_min_k4 (qmv_model.cpp:72-77)
            int s6, m6;
            if (j < 4) {
                s6 = sc(j) & 63;
                m6 = sc(j + 4) & 63;
            } else {
                s6 = (sc(j + 4) & 15) | ((sc(j - 4) >> 6) << 4);
                m6 = (sc(j + 4) >> 4) | ((sc(j) >> 6) << 4);
            }
            const int q0 = 4 + 8 * (j >> 1);
            const int sh = 4 * (j & 1);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[8 * j + i] = (w[q0 + i] >> sh) & kLo;
            ws[(j * 2) * kRows + t] = d * float(s6);
            ws[(j * 2 + 1) * kRows + t] = dmin * float(m6);
        }
    }
    tmem_st<kAColsPerStage>(tmem_a, a);
}

// The batch's activation blocks of one stage (act: a 288-byte row of eight
// Q8_1 blocks per column) into the B tiles (column c of block j at canon(c,
// .) of tile j) and the activation scales (xs: [kBlocks][2][kCols]).  Item
// t < batch x 8 is column t / 8's block t % 8; the tiles' rows past the batch
// stay zero from the kernel's start.
template <int TYPE>
__device__ __forceinline__ void convert_activations(const uint8_t* act, uint8_t* B, float* xs, int batch, int t) {
    const int c = t >> 3, j = t & 7;
    if (c >= batch) return;
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(act + c * kActRow + j * 36);
    const uint32_t ds = x32[0];
    const uint4 q0 = make_uint4(x32[1], x32[2], x32[3], x32[4]);
    const uint4 q1 = make_uint4(x32[5], x32[6], x32[7], x32[8]);
    float mx = 0.f;
    if constexpr (TYPE == P100_Q4_0) {
        mx = -8.0f * half_hi(ds);
    } else if constexpr (TYPE == P100_Q4_K) {
        int sq = 0;
        sq = __dp4a(int(q0.x), 0x01010101, sq);
        sq = __dp4a(int(q0.y), 0x01010101, sq);
        sq = __dp4a(int(q0.z), 0x01010101, sq);
        sq = __dp4a(int(q0.w), 0x01010101, sq);
        sq = __dp4a(int(q1.x), 0x01010101, sq);
        sq = __dp4a(int(q1.y), 0x01010101, sq);
        sq = __dp4a(int(q1.z), 0x01010101, sq);
        sq = __dp4a(int(q1.w), 0x01010101, sq);
        mx = float(sq);
    }
    *reinterpret_cast<uint4*>(B + j * kBTile + canon(c, 0)) = q0;
    *reinterpret_cast<uint4*>(B + j * kBTile + canon(c, 1)) = q1;
    xs[(j * 2) * kCols + c] = half_lo(ds);
    xs[(j * 2 + 1) * kCols + c] = mx;
}

// ------------------------------------------------------------ the kernel
// Shared memory: mbarriers at 0, two words at 240, the warpgroup / split-K
// exchange area [kCols][kRows] floats at kRedOff, the operand slots at kOpOff,
// the raw weight ring after them (slots raw_stride bytes apart), then the
// activation ring (raw_slots x kActBytes).
constexpr int kRedOff = 256;
constexpr int kOpOff = 9216;
constexpr int kRawOff = kOpOff + kOpSlots * kOpBytes;   // 62464, 1024-byte aligned
__host__ __device__ constexpr int raw_stride(int raw_bytes) { return (raw_bytes + 1023) & ~1023; }

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// v into the shared-memory word of cluster CTA `rank` that corresponds to
// this CTA's `local` (a store: no round trip).
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Columns 0..NC-1 of NB consecutive blocks of a warpgroup's tile in one
// stage, and the bias written back into them.
template <int NC, int NB>
__device__ __forceinline__ void epi_load(uint32_t acc, uint32_t (&v)[NB * NC]) {
#pragma unroll
    for (int jj = 0; jj < NB; ++jj)
        tmem_ld<NC>(acc + uint32_t(jj * kCols), *reinterpret_cast<uint32_t(*)[NC]>(v + jj * NC));
}
template <int NC, int NB>
__device__ __forceinline__ void epi_rebias(uint32_t acc) {
    if constexpr (NC == kCols && NB == 4) {
        tmem_fill<4 * kCols>(acc, kBias);
    } else {
#pragma unroll
        for (int jj = 0; jj < NB; ++jj) tmem_fill<NC>(acc + uint32_t(jj * kCols), kBias);
    }
}

// Grid: (slices x row tiles); cluster (slices, 1, 1) when slices > 1.  NC:
// the columns the epilogue reads (4, 8 or 16, at least the batch).
template <int TYPE, int NC>
__global__ void __launch_bounds__(kThreads, 1) qmv_tc_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* raw_empty = raw_full + kMaxRaw;
    uint64_t* op_full = raw_empty + kMaxRaw;
    uint64_t* op_free = op_full + kOpSlots;
    uint64_t* mma_done = op_free + kOpSlots;
    uint64_t* tmem_free = mma_done + kTmemStages;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + 240);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 244);
    static_assert((2 * kMaxRaw + 2 * kOpSlots + 2 * kTmemStages) * 8 <= 240, "barrier area");
    float* red = reinterpret_cast<float*>(smem + kRedOff);
    uint8_t* ops = smem + kOpOff;
    uint8_t* raws = smem + kRawOff;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == kProducerWarp && lane == 0) {   // the descriptors load while the block sets up
        prefetch_tensormap(&p.tmw);
        prefetch_tensormap(&p.tmx);
    }
    const int slice = p.slices > 1 ? static_cast<int>(cluster_rank()) : 0;
    const int row0 = static_cast<int>(blockIdx.x / p.slices) * kRows;
    const int groups = p.k / 256;
    const int g0 = groups * slice / p.slices, g1 = groups * (slice + 1) / p.slices;
    const int nst = g1 - g0;
    const int R = p.raw_slots, stride = raw_stride(p.raw_bytes);
    uint8_t* acts = raws + size_t(R) * stride;

    if (tid == 0) {
        for (int i = 0; i < R; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kConvWarps);
        }
        for (int i = 0; i < kOpSlots; ++i) {
            mbar_init(&op_full[i], kConvWarps);
            mbar_init(&op_free[i], kEpiWarps);
        }
        for (int i = 0; i < kTmemStages; ++i) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&tmem_free[i], kEpiWarps);
        }
        *s_abort = 0;
        fence_barrier_init();
    }
    // B tiles and activation scales of every slot zeroed: the rows and
    // columns past the batch are never written again
    for (int i = tid; i < kOpSlots * (kOpWs / 16); i += kThreads)
        *reinterpret_cast<uint4*>(ops + (i / (kOpWs / 16)) * kOpBytes + kOpB + (i % (kOpWs / 16)) * 16) =
            make_uint4(0u, 0u, 0u, 0u);
    constexpr int kXs16 = (kOpBytes - kOpXs) / 16;
    for (int i = tid; i < kOpSlots * kXs16; i += kThreads)
        *reinterpret_cast<uint4*>(ops + (i / kXs16) * kOpBytes + kOpXs + (i % kXs16) * 16) = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the zero rows, for the tensor core's reads
    if (warp == kMmaWarp) {   // tensor memory: kTmemCols columns, address into s_tmem
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(s_tmem)),
                     "r"(uint32_t(kTmemCols))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    pdl_allow_dependents();

    const bool epi = warp >= kConvWarps && warp < kConvWarps + kEpiWarps;
    const int wg = (warp - kConvWarps) >> 2;   // epilogue warpgroup: blocks 4 wg .. 4 wg + 3 of a stage
    const int r = (warp & 3) * 32 + lane;      // converters and epilogue: the row (tensor-memory lane)
    const uint32_t lanes = uint32_t((warp & 3) * 32) << 16;
    float y[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) y[c] = 0.f;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            const uint32_t tx = uint32_t(p.raw_bytes + kActRow * p.batch);
            // the first stages' weights go out before the previous kernel ends
            // (weights never depend on it), their activations after
            const int pre = min(R, nst);
            for (int s = 0; s < pre; ++s) {
                mbar_arrive_expect_tx(&raw_full[s], tx);
                tma_load_2d(raws + size_t(s) * stride, &p.tmw, (g0 + s) * (p.group_bytes / 2), row0, &raw_full[s],
                            policy);
            }
            pdl_wait_prior_grid();
            for (int s = 0; s < pre; ++s)
                tma_load_2d(acts + size_t(s) * kActBytes, &p.tmx, (g0 + s) * (kActRow / 2), 0, &raw_full[s], policy);
            int issued = pre;
            for (int s = pre; s < nst; ++s) {
                const int rs = s % R;
                if (!tc_wait(&raw_empty[rs], ((s / R) - 1) & 1, s_abort)) break;
                mbar_arrive_expect_tx(&raw_full[rs], tx);
                tma_load_2d(raws + size_t(rs) * stride, &p.tmw, (g0 + s) * (p.group_bytes / 2), row0, &raw_full[rs],
                            policy);
                tma_load_2d(acts + size_t(rs) * kActBytes, &p.tmx, (g0 + s) * (kActRow / 2), 0, &raw_full[rs],
                            policy);
                issued = s + 1;
            }
            // no copy may still be writing shared memory when the block exits
            for (int s = max(0, issued - R); s < issued; ++s) mbar_wait(&raw_full[s % R], (s / R) & 1);
        }
    } else if (warp < kConvWarps) {
        for (int s = 0; s < nst; ++s) {
            const int rs = s % R, os = s % kOpSlots;
            uint8_t* op = ops + size_t(os) * kOpBytes;
            bool ok = tc_wait(&raw_full[rs], (s / R) & 1, s_abort);
            // operand stage os (A, B tiles, scales) is free once the epilogue
            // is done with stage s - 4
            if (ok && s >= kOpSlots) ok = tc_wait(&op_free[os], ((s / kOpSlots) - 1) & 1, s_abort);
            if (__any_sync(0xffffffffu, !ok)) break;
            tc_fence_after();
            convert_weights<TYPE>(raws + size_t(rs) * stride, reinterpret_cast<float*>(op + kOpWs),
                                  tmem + lanes + uint32_t(kACol + os * kAColsPerStage), r);
            // activation items spread over the four warps' first lanes
            convert_activations<TYPE>(acts + size_t(rs) * kActBytes, op + kOpB, reinterpret_cast<float*>(op + kOpXs),
                                      p.batch, lane * kConvWarps + warp);
            tmem_wait_st();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // B tiles, for the tensor core's reads
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&raw_empty[rs]);
                mbar_arrive(&op_full[os]);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(TYPE == P100_Q8_0, true);
            int issued = 0;
            for (int s = 0; s < nst; ++s) {
                const int pp = s & 1, os = s % kOpSlots;
                bool ok = tc_wait(&op_full[os], (s / kOpSlots) & 1, s_abort);
                // accumulator stage pp biased: initially, then by the
                // epilogue of stage s - 2 after reading it
                if (ok) ok = tc_wait(&tmem_free[pp], (s >> 1) & 1, s_abort);
                if (!ok) break;
                tc_fence_after();
                const uint32_t bsm = smem_addr(ops + size_t(os) * kOpBytes + kOpB);
#pragma unroll
                for (int j = 0; j < kBlocks; ++j)
                    mma_i8_ts(tmem + uint32_t((pp * kBlocks + j) * kCols),
                              tmem + uint32_t(kACol + os * kAColsPerStage + j * 8), umma_desc(bsm + j * kBTile, 128, 256),
                              idesc);
                mma_commit(&mma_done[pp]);
                issued = s + 1;
            }
            // every MMA completes before the block frees tensor memory
            for (int s = max(0, issued - kTmemStages); s < issued; ++s) mbar_wait(&mma_done[s & 1], (s >> 1) & 1);
        }
        __syncwarp();
    } else if (epi) {
        using namespace qmvm;
        const uint32_t acc0 = tmem + lanes + uint32_t(4 * wg * kCols);
        // both accumulator stages start biased
        epi_rebias<NC, 4>(acc0);
        epi_rebias<NC, 4>(acc0 + uint32_t(kBlocks * kCols));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&tmem_free[0]);
            mbar_arrive(&tmem_free[1]);
        }
        // y may have been written by the previous kernel
        pdl_wait_prior_grid();
        const uint64_t neg_bias = pk(-12582912.0f, -12582912.0f);   // -1.5 * 2^23
        uint64_t y2[NC / 2];
#pragma unroll
        for (int c = 0; c < NC / 2; ++c) y2[c] = 0;
        for (int s = 0; s < nst; ++s) {
            const int pp = s & 1;
            const uint8_t* op = ops + size_t(s % kOpSlots) * kOpBytes;
            const bool ok = tc_wait(&mma_done[pp], (s >> 1) & 1, s_abort);
            if (__any_sync(0xffffffffu, !ok)) break;
            tc_fence_after();
            const uint32_t acc = acc0 + uint32_t(pp * kBlocks * kCols);
            const float* ws = reinterpret_cast<const float*>(op + kOpWs);
            const float* xs = reinterpret_cast<const float*>(op + kOpXs);
            // the four blocks in passes of kNB (16 columns: two passes of 32
            // registers, so the dots and sums stay in registers)
            constexpr int kNB = NC == kCols ? 2 : 4;
#pragma unroll
            for (int h0 = 0; h0 < 4; h0 += kNB) {
                uint32_t v[kNB * NC];
                epi_load<NC, kNB>(acc + uint32_t(h0 * kCols), v);
                tmem_wait_ld();
                epi_rebias<NC, kNB>(acc + uint32_t(h0 * kCols));
#pragma unroll
                for (int jb = 0; jb < kNB; ++jb) {
                    const int j = 4 * wg + h0 + jb;
                    const float w0 = ws[(j * 2) * kRows + r];
                    const uint64_t w02 = pk(w0, w0);
                    const float w1 = TYPE == P100_Q4_K ? ws[(j * 2 + 1) * kRows + r] : 0.f;
                    const uint64_t w12 = pk(w1, w1);
                    const float4* dx4 = reinterpret_cast<const float4*>(xs + (j * 2) * kCols);
                    const float4* mx4 = reinterpret_cast<const float4*>(xs + (j * 2 + 1) * kCols);
#pragma unroll
                    for (int c4 = 0; c4 < NC / 4; ++c4) {
                        const float4 d = dx4[c4], m = mx4[c4];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int c2 = 2 * c4 + h;
                            const uint64_t dv = h ? pk(d.z, d.w) : pk(d.x, d.y);
                            const uint64_t mv = h ? pk(m.z, m.w) : pk(m.x, m.y);
                            const uint64_t dot =
                                add2(pk_bits(int(v[jb * NC + 2 * c2]), int(v[jb * NC + 2 * c2 + 1])), neg_bias);
                            if constexpr (TYPE == P100_Q4_0) {
                                // d_w * (d_x * dot - 8 * sum_x), the q81 block formula
                                y2[c2] = fma2(w02, fma2(dot, dv, mv), y2[c2]);
                            } else if constexpr (TYPE == P100_Q8_0) {
                                y2[c2] = fma2(mul2(w02, dv), dot, y2[c2]);
                            } else {
                                // (d sc) d_x dot - (dmin mn) d_x sum(q)
                                y2[c2] = fma2(mul2(w02, dv), dot, y2[c2]);
                                y2[c2] = fma2(mul2(w12, dv) ^ 0x8000000080000000ull, mv, y2[c2]);
                            }
                        }
                    }
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tmem_free[pp]);
                mbar_arrive(&op_free[s % kOpSlots]);
            }
        }
#pragma unroll
        for (int c2 = 0; c2 < NC / 2; ++c2) {
            const float2 f = unpk(y2[c2]);
            y[2 * c2] = f.x;
            y[2 * c2 + 1] = f.y;
        }
    }

    // the two epilogue warpgroups' sums: the second's into the first's (in
    // the exchange area), then the split K's slice partials in slice order:
    // once every CTA of the cluster is done with its ring, slices 1.. store
    // their partials into slice 0's raw ring (distributed shared memory,
    // stores only), and slice 0 adds them after the second cluster barrier
    __syncthreads();
    if (epi && wg == 1)
#pragma unroll
        for (int c = 0; c < NC; ++c) red[c * kRows + r] = y[c];
    __syncthreads();
    const bool lead = epi && wg == 0;
    if (lead)
#pragma unroll
        for (int c = 0; c < NC; ++c) y[c] += red[c * kRows + r];
    if (p.slices > 1) {
        float* recv = reinterpret_cast<float*>(raws);   // [slices - 1][NC][kRows]
        qmvm::cluster_sync_all();
        if (lead && slice > 0)
#pragma unroll
            for (int c = 0; c < NC; ++c) st_cluster_f32(recv + ((slice - 1) * NC + c) * kRows + r, 0u, y[c]);
        qmvm::cluster_sync_all();
        if (lead && slice == 0)
            for (int sl = 1; sl < p.slices; ++sl)
#pragma unroll
                for (int c = 0; c < NC; ++c) y[c] += recv[((sl - 1) * NC + c) * kRows + r];
    }
    if (lead && slice == 0 && row0 + r < p.rows && !*s_abort)
#pragma unroll
        for (int c = 0; c < NC; ++c)
            if (c < p.batch) p.y[size_t(c) * p.rows + row0 + r] = y[c];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(kTmemCols))
                     : "memory");
}
}  // namespace qmvtc
}  // namespace p100b
