// common.cuh — shared device helpers for the sm_100a kernels of p100_b200.
//
// Everything here is hand-written inline PTX or plain CUDA: mbarriers and
// untiled bulk-async copies (global -> this CTA's shared memory only), bounded
// waits on %globaltimer, and the per-device flag that a timed-out wait sets.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "p100/b200.h"

namespace p100b {

// ------------------------------------------------------------ host helpers
// Implemented in capi.cu.
p100_status set_error(p100_status status, const char* fmt, ...);
p100_status cuda_status(cudaError_t err, const char* what);
void clear_error();
// P100_OK when the current device is an sm_100 part (cached per device).
p100_status require_sm100(int* device_out, int* sm_count_out);

// ------------------------------------------------------------ device state
// Set to kDevErrTimeout by any bounded wait that runs out; read by
// p100_device_error().  The library is one CUDA translation unit (capi.cu),
// so this definition exists once per device module.
__device__ int g_device_error = 0;
constexpr int kDevErrTimeout = 1;
constexpr int kDevErrInput = 2;    // a device-resident index (token, position) out of range
// One second: far above any legitimate wait in these kernels (microseconds).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the barrier phase with the given parity to complete, for at most
// kWaitLimitNs.  Returns false (and raises the device flag) when it gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicExch(&g_device_error, kDevErrTimeout);
            return false;
        }
    }
}

// ------------------------------------------------------------ bulk copies
// L2 policy for data read exactly once (weights, KV): evict first, so the
// small re-read operands (activations, partials) keep their lines.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// Untiled bulk-async copy global -> this CTA's shared memory, completing on
// `bar` with `bytes` transaction bytes.  dst, src 16-byte aligned; bytes a
// multiple of 16.  One destination CTA; the source is always this GPU's memory.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Tiled tensor copy global -> this CTA's shared memory, completing on `bar`:
// the box of the 4-d tensor map at coordinates (c0, c1, c2, c3), elements
// outside the tensor read as zero.  c0 * element size must be a multiple of
// 16 bytes and no coordinate negative; dst aligned as the map's swizzle wants
// (1024 bytes for the 128-byte swizzle).  One destination CTA.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Starts fetching a TMA tensor map (a __grid_constant__ kernel parameter) so
// that the first copy through it does not wait for the descriptor.
__device__ __forceinline__ void prefetch_tensormap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------ programmatic dependent launch
// Both are no-ops for a kernel launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_allow_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ small math
__device__ __forceinline__ float half_lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}
// Bytes 2..5 of the 8-byte pair (lo, hi): realigns a 2-byte-offset word.
__device__ __forceinline__ uint32_t shift2(uint32_t lo, uint32_t hi) { return __byte_perm(lo, hi, 0x5432); }

// fp16 of v (nearest even) into the 2-byte aligned p with one 16-bit store.
// The scale of a K/V block appended inside the attention kernel is written
// while other CTAs of the same head read neighbouring rows with bulk copies
// (async proxy); written as two 8-bit stores, its low byte read back as 0
// (reproduced: the quantised-cache decoder test fails with the two-store
// form and passes with this one, while the same two-store form is exact in
// init_kv_quant_kernel, where no copy reads the rows).  One store keeps the
// two bytes together.
__device__ __forceinline__ void store_half_bits(uint8_t* p, float v) {
    *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

}  // namespace p100b
