// capi.cu — the extern "C" entry points of include/p100/b200.h for the
// quantised mat-vec and FlashAttention decode paths, plus library plumbing
// (status text, device checks, the bounded-wait flag).
//
// Single CUDA translation unit: every kernel header is included here so the
// library has one device module and one g_device_error word per device.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "fa_decode.cuh"
#include "fa_mma.cuh"
#include "h16.cuh"
#include "qmv.cuh"
#include "qmv_mma.cuh"
#include "qmv_tc.cuh"
#include "qmv_team.cuh"
#include "quant.cuh"

namespace p100b {

namespace {
thread_local std::string t_error;
std::mutex g_dev_mutex;
int g_dev_sm100[64];     // 0 unknown, 1 sm_100, -1 other
int g_dev_sms[64];
}  // namespace

p100_status set_error(p100_status status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_error = buf;
    return status;
}

void clear_error() { t_error.clear(); }

p100_status cuda_status(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return P100_OK;
    return set_error(P100_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

p100_status require_sm100(int* device_out, int* sm_count_out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return set_error(P100_ERR_UNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(err));
    }
    if (dev < 0 || dev >= 64) return set_error(P100_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (g_dev_sm100[dev] == 0) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            (void)cudaGetLastError();
            return set_error(P100_ERR_UNSUPPORTED, "cannot query device %d", dev);
        }
        g_dev_sm100[dev] = (major == 10 && minor == 0) ? 1 : -1;
        g_dev_sms[dev] = sms;
    }
    if (g_dev_sm100[dev] != 1)
        return set_error(P100_ERR_UNSUPPORTED, "device %d is not sm_100; this build has sm_100a code only", dev);
    if (device_out) *device_out = dev;
    if (sm_count_out) *sm_count_out = g_dev_sms[dev];
    return P100_OK;
}

namespace {

// the reference's three formats (every kernel) and ggml's Q5_K / Q6_K (the
// general mat-vec and dequantisation kernels)
bool ref_type(int t) { return t == P100_Q4_0 || t == P100_Q8_0 || t == P100_Q4_K; }
bool known_type(int t) { return ref_type(t) || t == P100_Q5_K || t == P100_Q6_K; }
int elems_of(int t) { return t == P100_Q4_0 || t == P100_Q8_0 ? 32 : 256; }
int bytes_of(int t) {
    return t == P100_Q4_0 ? 18 : t == P100_Q8_0 ? 34 : t == P100_Q4_K ? 144 : t == P100_Q5_K ? 176 : 210;
}

p100_status launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

// SM count of a device that require_sm100 has seen.
int sms_of(int dev) { return dev >= 0 && dev < 64 ? g_dev_sms[dev] : 0; }

// ------------------------------------------------------------------ qmv plan
struct QmvPlan {
    qmv::Params p{};
    int bmax = 0, grid = 0, threads = 0;
    size_t smem = 0;
};

size_t round128(size_t x) { return (x + 127) & ~size_t(127); }

// Fills plan for the bulk path with up to bmax activation columns per launch;
// false if the shape or alignment needs the generic kernel.  Stages are whole
// rows, about 16 KB; for one column the CTA keeps to half an SM's shared
// memory so two launches of a chain are resident together.
constexpr size_t kStageTarget = 16 * 1024;

bool plan_bulk(int type, const void* w, int rows, int k, int batch, int sms, QmvPlan& plan) {
    if (!ref_type(type)) return false;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    if (reinterpret_cast<uintptr_t>(w) % 16 || row_bytes % 16 || k % 256) return false;
    const int rps = int(std::max<size_t>(1, std::min<size_t>(qmv::kMaxRows, (kStageTarget + row_bytes / 2) / row_bytes)));
    const size_t slot = round128(size_t(rps) * row_bytes);
    for (int bmax = std::min(4, batch); bmax >= 1; --bmax) {
        const size_t limit = bmax == 1 ? size_t(qmv::kSmemLimit) / 2 - 1024 : size_t(qmv::kSmemLimit);
        const size_t part_off = 512;                                       // barriers + tickets
        const size_t part_bytes = size_t(qmv::kMaxSlots) * qmv::kConsumers * qmv::kMaxRows * bmax * 4;
        const size_t codes_off = part_off + round128(part_bytes);
        const size_t meta_off = codes_off + round128(size_t(bmax) * k);    // codes: bmax*8*(k/32) words
        const size_t ring_off = meta_off + round128(size_t(bmax) * (k / 32) * 8);
        if (ring_off + 3 * slot > limit) continue;
        const int nslot = int(std::min<size_t>(qmv::kMaxSlots, (limit - ring_off) / slot));
        plan.p.rows = rows;
        plan.p.k = k;
        plan.p.row_bytes = int(row_bytes);
        plan.p.ipr = k / 64;
        plan.p.rps = rps;
        plan.p.nslot = nslot;
        plan.p.slot_bytes = int(slot);
        plan.p.part_off = int(part_off);
        plan.p.codes_off = int(codes_off);
        plan.p.meta_off = int(meta_off);
        plan.p.ring_off = int(ring_off);
        plan.bmax = bmax;
        plan.smem = ring_off + size_t(nslot) * slot;
        plan.threads = qmv::kThreads;
        plan.grid = std::max(1, std::min(sms, (rows + rps - 1) / rps));
        return true;
    }
    return false;
}

template <int TYPE, int B>
p100_status launch_bulk_t(const QmvPlan& plan, bool pdl, cudaStream_t stream) {
    auto kern = qmv::qmv_bulk_kernel<TYPE, B>;
    static thread_local int configured_smem[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_smem[dev] < int(plan.smem)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, qmv::kSmemLimit);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(qmv)");
        configured_smem[dev] = qmv::kSmemLimit;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(plan.threads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, plan.p), "qmv_bulk_kernel launch");
}

template <int TYPE>
p100_status launch_bulk_type(const QmvPlan& plan, int cols, bool pdl, cudaStream_t s) {
    switch (cols) {
        case 1: return launch_bulk_t<TYPE, 1>(plan, pdl, s);
        case 2: return launch_bulk_t<TYPE, 2>(plan, pdl, s);
        case 3: return launch_bulk_t<TYPE, 3>(plan, pdl, s);
        default: return launch_bulk_t<TYPE, 4>(plan, pdl, s);
    }
}

// ------------------------------------------------------------------ team plan
struct TeamPlan {
    qmvt::Params p{};
    int grid = 0;
    size_t smem = 0;
};

// The batch-1 kernel: a lane per 256-weight column group, one row per team
// per stage.  Needs 16-byte aligned weights and activations and k % 256 == 0.
bool plan_team(int type, const void* w, const void* xq, int rows, int k, int batch, int sms, TeamPlan& plan) {
    if (!known_type(type)) return false;
    if (batch != 1 || k % 256 || reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(xq) % 16)
        return false;
    const int ngroups = k / 256;
    const int team = qmvt::team_lanes(ngroups);
    // teams of several warps meet at a named barrier of team lanes: every
    // consumer lane must belong to a whole team (a team of 96 lanes would
    // leave 64 lanes waiting at a barrier that never fills)
    if (team > qmvt::kConsumers * 32 || (qmvt::kConsumers * 32) % team) return false;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    // Stages are 16-byte bulk copies: rows of whole 16-byte units, or (Q6_K,
    // whose groups are read on the 2-byte grid) a matrix that ends on the
    // grid, each stage widened to it (up to 14 bytes before its first row and
    // 14 after its last, and the last group's reads 6 past it: 32 more bytes
    // per slot).
    const bool ragged = row_bytes % 16 != 0;
    if (ragged && (type != P100_Q6_K || (size_t(rows) * row_bytes) % 16)) return false;
    // Q6_K groups are read as aligned words that run up to 6 bytes past the group
    const size_t tail = type == P100_Q6_K ? 16 : 0;
    const int teams = qmvt::kConsumers * 32 / team;
    const size_t slot = round128(size_t(teams) * row_bytes + (ragged ? 32 : 0));
    const size_t part_off = 384;   // 2 x 8 ring mbarriers + the activation one; the fused norm's partials at 256
    const size_t act_off = part_off + round128(size_t(2) * teams * std::max(1, team / 32) * 4);
    const size_t ring_off = act_off + round128(size_t(k / 32) * 36);   // the Q8_1 row
    if (ring_off + 2 * slot + tail > size_t(qmvt::kSmemLimit)) return false;
    const int nslot = int(std::min<size_t>(qmvt::kMaxSlots, (qmvt::kSmemLimit - ring_off - tail) / slot));
    plan.p.rows = rows;
    plan.p.k = k;
    plan.p.row_bytes = int(row_bytes);
    plan.p.ngroups = ngroups;
    plan.p.team = team;
    plan.p.teams = teams;
    plan.p.nslot = nslot;
    plan.p.slot_bytes = int(slot);
    plan.p.part_off = int(part_off);
    plan.p.act_off = int(act_off);
    plan.p.ring_off = int(ring_off);
    plan.smem = ring_off + size_t(nslot) * slot + tail;
    plan.grid = std::max(1, std::min(sms, (rows + teams - 1) / teams));
    return true;
}

template <int TYPE, int NG, bool PUSH = false>
p100_status launch_team_t(const TeamPlan& plan, bool pdl, cudaStream_t stream) {
    auto kern = qmvt::qmv_team_kernel<TYPE, NG, PUSH>;
    static thread_local int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, qmvt::kSmemLimit);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(qmv_team)");
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(qmvt::kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, plan.p), "qmv_team_kernel launch");
}

// Kernels compiled for the hidden sizes of the Llama-3 8B/70B decode shapes
// (k = 4096, 8192, 14336, 28672); any other k % 256 == 0 takes NG = 0.
template <int TYPE, bool PUSH = false>
p100_status launch_team_type(const TeamPlan& plan, int batch, bool pdl, cudaStream_t s) {
    (void)batch;   // the team kernel serves one column
    switch (plan.p.ngroups) {
        case 16: return launch_team_t<TYPE, 16, PUSH>(plan, pdl, s);
        case 32: return launch_team_t<TYPE, 32, PUSH>(plan, pdl, s);
        case 56: return launch_team_t<TYPE, 56, PUSH>(plan, pdl, s);
        case 112: return launch_team_t<TYPE, 112, PUSH>(plan, pdl, s);
        default: return launch_team_t<TYPE, 0, PUSH>(plan, pdl, s);
    }
}

// ------------------------------------------------------------------ batched plan
using MmaKernel = void (*)(qmvm::Params);

MmaKernel mma_kernel(int type, int bpw, int ncg) {
#define P100_MMA_BPW(T, N)                                  \
    switch (bpw) {                                          \
        case 2: return qmvm::qmv_mma_kernel<T, 2, N>;       \
        case 4: return qmvm::qmv_mma_kernel<T, 4, N>;       \
        case 8: return qmvm::qmv_mma_kernel<T, 8, N>;       \
        case 16: return qmvm::qmv_mma_kernel<T, 16, N>;     \
        case 32: return qmvm::qmv_mma_kernel<T, 32, N>;     \
        default: return nullptr;                            \
    }
#define P100_MMA_BPW_K(N)                                   \
    switch (bpw) {                                          \
        case 8: return qmvm::qmv_mma_kernel<P100_Q4_K, 8, N>;   \
        case 16: return qmvm::qmv_mma_kernel<P100_Q4_K, 16, N>; \
        case 32: return qmvm::qmv_mma_kernel<P100_Q4_K, 32, N>; \
        default: return nullptr;                            \
    }
    if (ncg == 1) {
        switch (type) {
            case P100_Q4_0: P100_MMA_BPW(P100_Q4_0, 1)
            case P100_Q8_0: P100_MMA_BPW(P100_Q8_0, 1)
            default: P100_MMA_BPW_K(1)
        }
    }
    switch (type) {
        case P100_Q4_0: P100_MMA_BPW(P100_Q4_0, 2)
        case P100_Q8_0: P100_MMA_BPW(P100_Q8_0, 2)
        default: P100_MMA_BPW_K(2)
    }
#undef P100_MMA_BPW
#undef P100_MMA_BPW_K
}

// The largest dynamic shared memory on every batched kernel, once per device;
// for a K split also the number of S-CTA clusters that fit the GPU at once.
bool mma_prepare(MmaKernel kern, int slices, int threads, int* max_clusters) {
    struct Entry { int dev; MmaKernel kern; int slices, threads, clusters; };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(mu);
    bool attr_done = false;
    for (const Entry& e : cache) {
        if (e.dev != dev || e.kern != kern) continue;
        attr_done = true;
        if (e.slices == slices && e.threads == threads) {
            *max_clusters = e.clusters;
            return true;
        }
    }
    if (!attr_done &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, qmvm::kSmemLimit) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    int clusters = 0;
    if (slices > 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(slices);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = qmvm::kSmemLimit;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = slices;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            clusters = 0;
        }
    }
    cache.push_back({dev, kern, slices, threads, clusters});
    *max_clusters = clusters;
    return true;
}

struct MmaPlan {
    qmvm::Params p{};
    MmaKernel kern = nullptr;
    int grid = 0, threads = 0;
    size_t smem = 0;
};

// Batch 2..16 on the tensor cores (every type): 16-byte aligned weights and
// activations, k % 256 == 0.  One column group of 8 up to batch 8, two
// above.  Picks the fewest K slices (CTAs per cluster), then the most
// consumer warps, whose per-warp share of blocks is compiled in and whose
// layout fits: two ring slots ahead of the activations.
bool plan_mma(int type, const void* w, const void* xq, int rows, int k, int batch, int sms, MmaPlan& plan) {
    if (!ref_type(type)) return false;
    if (batch < 2 || batch > 16 || !known_type(type)) return false;
    if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(xq) % 16 || k % 256) return false;
    const int nb = k / 32;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    const int rows_per_stage = qmvm::stage_rows(type);
    const int ncg = batch > 8 ? 2 : 1;   // column groups of 8
    for (int slices : {1, 2, 4, 8}) {
        for (int nw = qmvm::kMaxConsumers; nw >= 4; --nw) {
            if (nb % (slices * nw)) continue;
            const int bpw = nb / (slices * nw);
            const int nbs = nw * bpw;
            const size_t slice = size_t(qmvm::slice_bytes_of(type, nbs));
            if (slice % 16 || (size_t(nbs) * 36) % 16) continue;
            const MmaKernel kern = mma_kernel(type, bpw, ncg);
            if (!kern) continue;
            const int threads = (nw + 1) * 32;
            if (threads > qmvm::max_threads(bpw, ncg)) continue;
            int max_clusters = 0;
            if (!mma_prepare(kern, slices, threads, &max_clusters)) continue;
            int nrb = (rows + rows_per_stage - 1) / rows_per_stage;
            nrb = std::min(nrb, slices == 1 ? sms : max_clusters);
            if (nrb < 1) continue;
            const size_t row_stride = slice + 16;   // padded: rows in distinct banks
            const size_t slot = round128(size_t(rows_per_stage) * row_stride);
            const size_t act_stride = size_t(nbs) * 36 + 16;
            const size_t act_bytes = size_t(batch) * act_stride;
            const size_t dm_off = 256;                                   // 2 x 8 ring mbarriers + 2
            const size_t part_off = dm_off + size_t(nbs) * 8 * 16;
            const size_t res_off = part_off + size_t(2) * nw * rows_per_stage * qmvm::kPartStride * 4;
            const size_t res_bytes = slices > 1 ? size_t((rows + nrb - 1) / nrb) * 16 * 4 : 0;
            const size_t scr_off = res_off + round128(res_bytes);
            const size_t scr_bytes = type == P100_Q4_K ? size_t(nw) * 16 * 8 * 16 : 0;
            const size_t ring_off = round128(scr_off + scr_bytes);
            if (ring_off + 3 * slot > size_t(qmvm::kSmemLimit)) continue;
            const int nslot = int(std::min<size_t>(qmvm::kMaxSlots, (qmvm::kSmemLimit - ring_off) / slot));
            const int act_slot = nslot - int((act_bytes + slot - 1) / slot);
            if (act_slot < 2) continue;   // the first two stages go ahead of the activations
            qmvm::Params& p = plan.p;
            p.rows = rows;
            p.k = k;
            p.batch = batch;
            p.consumers = nw;
            p.slices = slices;
            p.row_bytes = int(row_bytes);
            p.slice_bytes = int(slice);
            p.row_stride = int(row_stride);
            p.act_stride = int(act_stride);
            p.nslot = nslot;
            p.slot_bytes = int(slot);
            p.act_slot = act_slot;
            p.dm_off = int(dm_off);
            p.part_off = int(part_off);
            p.res_off = int(res_off);
            p.scr_off = int(scr_off);
            p.ring_off = int(ring_off);
            plan.kern = kern;
            plan.grid = nrb * slices;
            plan.threads = threads;
            plan.smem = ring_off + size_t(nslot) * slot;
            return true;
        }
    }
    return false;
}

p100_status launch_mma(const MmaPlan& plan, bool pdl, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(plan.threads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (plan.p.slices > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = plan.p.slices;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cuda_status(cudaLaunchKernelEx(&cfg, plan.kern, plan.p), "qmv_mma_kernel launch");
}

// ------------------------------------------------------------------ tensor-core (tcgen05) batched plan
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

struct TcPlan {
    qmvtc::Params p{};
    int grid = 0;
    size_t smem = 0;
};

// Batch 2..16 of Q4_0, Q8_0 or Q4_K with 16-byte aligned rows of whole
// 256-value groups: row tiles of 128, the K split over a cluster of up to 8
// CTAs while the grid stays within the SMs, raw stages in the ring as shared
// memory allows.
bool plan_tc(int type, const void* w, const void* xq, int rows, int k, int batch, int sms, TcPlan& plan) {
    if (!ref_type(type) || batch < 2 || batch > qmvtc::kCols || k % 256 || rows <= 0) return false;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    if (reinterpret_cast<uintptr_t>(w) % 16 || row_bytes % 16 || reinterpret_cast<uintptr_t>(xq) % 16) return false;
    const int groups = k / 256;
    const int group_bytes = static_cast<int>(row_bytes / size_t(groups));
    const int tiles = (rows + qmvtc::kRows - 1) / qmvtc::kRows;
    int slices = 1;
    while (slices < 8 && tiles * slices * 2 <= sms && groups / (slices * 2) >= 2) slices *= 2;
    const int raw_bytes = qmvtc::kRows * group_bytes;
    const int slot_all = qmvtc::raw_stride(raw_bytes) + qmvtc::kActBytes;   // weights + activations of a stage
    const int slots = std::min(qmvtc::kMaxRaw, (qmvtc::kSmemLimit - qmvtc::kRawOff) / slot_all);
    if (slots < 2) return false;
    // slice 0 receives the other slices' partial sums in its raw ring
    while (slices > 1 && size_t(slices - 1) * qmvtc::kCols * qmvtc::kRows * 4 >
                             size_t(slots) * size_t(qmvtc::raw_stride(raw_bytes)))
        slices /= 2;
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {cuuint64_t(row_bytes / 2), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
    const cuuint32_t box[2] = {cuuint32_t(group_bytes / 2), cuuint32_t(qmvtc::kRows)};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&plan.p.tmw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    // the Q8_1 rows: a stage's eight blocks of the batch's columns per box
    const size_t xrow = size_t(k / 32) * 36;
    const cuuint64_t xdims[2] = {cuuint64_t(xrow / 2), cuuint64_t(batch)};
    const cuuint64_t xstrides[1] = {cuuint64_t(xrow)};
    const cuuint32_t xbox[2] = {cuuint32_t(qmvtc::kActRow / 2), cuuint32_t(batch)};
    if (encode(&plan.p.tmx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(xq), xdims, xstrides, xbox, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    plan.p.xq = static_cast<const uint8_t*>(xq);
    plan.p.rows = rows;
    plan.p.k = k;
    plan.p.batch = batch;
    plan.p.slices = slices;
    plan.p.raw_slots = slots;
    plan.p.raw_bytes = raw_bytes;
    plan.p.group_bytes = group_bytes;
    plan.grid = tiles * slices;
    plan.smem = size_t(qmvtc::kRawOff) + size_t(slots) * slot_all;
    return true;
}

template <int TYPE, int NC>
p100_status launch_tc_t(const TcPlan& plan, bool pdl, cudaStream_t stream) {
    auto kern = qmvtc::qmv_tc_kernel<TYPE, NC>;
    static thread_local int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, qmvtc::kSmemLimit);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(qmv_tc)");
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(qmvtc::kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (plan.p.slices > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = plan.p.slices;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, plan.p), "qmv_tc_kernel launch");
}

// The epilogue reads 4, 8 or 16 of the 16 accumulator columns: the fewest
// that hold the batch.
template <int TYPE>
p100_status launch_tc_cols(const TcPlan& plan, bool pdl, cudaStream_t s) {
    if (plan.p.batch <= 4) return launch_tc_t<TYPE, 4>(plan, pdl, s);
    if (plan.p.batch <= 8) return launch_tc_t<TYPE, 8>(plan, pdl, s);
    return launch_tc_t<TYPE, 16>(plan, pdl, s);
}

p100_status launch_tc(int type, const TcPlan& plan, bool pdl, cudaStream_t s) {
    switch (type) {
        case P100_Q4_0: return launch_tc_cols<P100_Q4_0>(plan, pdl, s);
        case P100_Q8_0: return launch_tc_cols<P100_Q8_0>(plan, pdl, s);
        default: return launch_tc_cols<P100_Q4_K>(plan, pdl, s);
    }
}

p100_status run_qmv(int type, const void* w, int rows, int k, const void* xq, int batch, float* y, unsigned flags,
                    cudaStream_t stream) {
    if (!known_type(type)) return set_error(P100_ERR_INVALID, "unknown weight type %d", type);
    if (k <= 0 || k % elems_of(type)) return set_error(P100_ERR_INVALID, "whole weight blocks required");
    if (rows < 0) return set_error(P100_ERR_INVALID, "rows must be non-negative");
    if (batch < 1 || batch > 16) return set_error(P100_ERR_INVALID, "batch must be in 1..16");
    if (rows == 0) return P100_OK;
    if (!w || !xq || !y) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(xq) % 4) return set_error(P100_ERR_INVALID, "x_q8_1 must be 4-byte aligned");
    if (reinterpret_cast<uintptr_t>(w) % 2) return set_error(P100_ERR_INVALID, "weights must be 2-byte aligned");
    int sms = 0;
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    const bool pdl = (flags & P100_QMV_PDL) != 0;
    TeamPlan tplan;
    if (plan_team(type, w, xq, rows, k, batch, sms, tplan)) {
        tplan.p.w = static_cast<const uint8_t*>(w);
        tplan.p.xq = static_cast<const uint8_t*>(xq);
        tplan.p.y = y;
        tplan.p.col0 = 0;
        switch (type) {
            case P100_Q4_0: return launch_team_type<P100_Q4_0>(tplan, batch, pdl, stream);
            case P100_Q8_0: return launch_team_type<P100_Q8_0>(tplan, batch, pdl, stream);
            case P100_Q4_K: return launch_team_type<P100_Q4_K>(tplan, batch, pdl, stream);
            case P100_Q5_K: return launch_team_type<P100_Q5_K>(tplan, batch, pdl, stream);
            default: return launch_team_type<P100_Q6_K>(tplan, batch, pdl, stream);
        }
    }
    // the tcgen05 kernel by default where it measured faster than mma.sync:
    // Q8_0 / Q4_K on large matrices (its fixed cost loses on small ones, and
    // Q4_0's nibble unpacking keeps it behind mma.sync at every size)
    const bool tc_default = (type == P100_Q8_0 || type == P100_Q4_K) && size_t(rows) * size_t(k) >= (size_t(1) << 25);
    const bool want_tc = (flags & P100_QMV_TC) || (tc_default && !(flags & P100_QMV_MMA));
    TcPlan tc;
    if (want_tc && plan_tc(type, w, xq, rows, k, batch, sms, tc)) {
        tc.p.y = y;
        return launch_tc(type, tc, pdl, stream);
    }
    MmaPlan mplan;
    if (plan_mma(type, w, xq, rows, k, batch, sms, mplan)) {
        mplan.p.w = static_cast<const uint8_t*>(w);
        mplan.p.xq = static_cast<const uint8_t*>(xq);
        mplan.p.y = y;
        return launch_mma(mplan, pdl, stream);
    }
    QmvPlan plan;
    if (plan_bulk(type, w, rows, k, batch, sms, plan)) {
        plan.p.w = static_cast<const uint8_t*>(w);
        plan.p.xq = static_cast<const uint8_t*>(xq);
        plan.p.y = y;
        for (int c0 = 0; c0 < batch; c0 += plan.bmax) {
            const int cols = std::min(plan.bmax, batch - c0);
            plan.p.col0 = c0;
            p100_status st;
            // Only the first launch may overlap the previous kernel; later
            // column chunks follow this call's own launches.
            const bool chained = pdl && c0 == 0;
            switch (type) {
                case P100_Q4_0: st = launch_bulk_type<P100_Q4_0>(plan, cols, chained, stream); break;
                case P100_Q8_0: st = launch_bulk_type<P100_Q8_0>(plan, cols, chained, stream); break;
                default: st = launch_bulk_type<P100_Q4_K>(plan, cols, chained, stream); break;
            }
            if (st) return st;
        }
        return P100_OK;
    }
    // Q5_K / Q6_K at batch 2..16 (no tensor-core form): one team-kernel
    // launch per column (col0), each streaming the whole matrix.  Measured
    // against the warp-per-row kernel, which re-reads every row per column
    // too, at 4096 x 14336: 4.2x faster at every batch from 2 to 16.
    if (!ref_type(type) && batch > 1 && plan_team(type, w, xq, rows, k, 1, sms, tplan)) {
        tplan.p.w = static_cast<const uint8_t*>(w);
        tplan.p.xq = static_cast<const uint8_t*>(xq);   // column c at c * k/32 * 36 bytes: 16-byte aligned
        tplan.p.y = y;
        for (int c = 0; c < batch; ++c) {
            tplan.p.col0 = c;
            // later columns only read what the earlier launches read
            const p100_status st = type == P100_Q5_K ? launch_team_type<P100_Q5_K>(tplan, 1, pdl || c > 0, stream)
                                                     : launch_team_type<P100_Q6_K>(tplan, 1, pdl || c > 0, stream);
            if (st) return st;
        }
        return P100_OK;
    }
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    const dim3 grid((rows + 7) / 8);
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const uint8_t* xb = static_cast<const uint8_t*>(xq);
    switch (type) {
        case P100_Q4_0: qmv::qmv_generic_kernel<P100_Q4_0><<<grid, 256, 0, stream>>>(wb, xb, y, rows, k, batch, row_bytes); break;
        case P100_Q8_0: qmv::qmv_generic_kernel<P100_Q8_0><<<grid, 256, 0, stream>>>(wb, xb, y, rows, k, batch, row_bytes); break;
        case P100_Q4_K: qmv::qmv_generic_kernel<P100_Q4_K><<<grid, 256, 0, stream>>>(wb, xb, y, rows, k, batch, row_bytes); break;
        case P100_Q5_K: qmv::qmv_generic_kernel<P100_Q5_K><<<grid, 256, 0, stream>>>(wb, xb, y, rows, k, batch, row_bytes); break;
        default: qmv::qmv_generic_kernel<P100_Q6_K><<<grid, 256, 0, stream>>>(wb, xb, y, rows, k, batch, row_bytes); break;
    }
    return launch_status("qmv_generic_kernel launch");
}

// Batch-1 mat-vec of a row-parallel matrix whose partial sums go straight
// into every rank's peer slots (the team kernel's push epilogue).  False
// when the team kernel does not take the shape (the caller then writes y and
// pushes separately).  ar: the exchange's PeerAr in device memory (ar_host:
// the same, on the host).
bool run_qmv_push(int type, const void* w, int rows, int k, const void* xq, const dec::PeerAr* ar,
                  const dec::PeerAr& ar_host, cudaStream_t stream, p100_status* st) {
    int sms = 0;
    *st = P100_OK;
    if (require_sm100(nullptr, &sms) || !known_type(type) || rows != ar_host.n) return false;
    TeamPlan tplan;
    if (!plan_team(type, w, xq, rows, k, 1, sms, tplan)) return false;
    tplan.p.w = static_cast<const uint8_t*>(w);
    tplan.p.xq = static_cast<const uint8_t*>(xq);
    tplan.p.y = nullptr;
    tplan.p.col0 = 0;
    tplan.p.ar = ar;
    switch (type) {
        case P100_Q4_0: *st = launch_team_type<P100_Q4_0, true>(tplan, 1, true, stream); break;
        case P100_Q8_0: *st = launch_team_type<P100_Q8_0, true>(tplan, 1, true, stream); break;
        case P100_Q4_K: *st = launch_team_type<P100_Q4_K, true>(tplan, 1, true, stream); break;
        case P100_Q5_K: *st = launch_team_type<P100_Q5_K, true>(tplan, 1, true, stream); break;
        default: *st = launch_team_type<P100_Q6_K, true>(tplan, 1, true, stream); break;
    }
    return true;
}

// Batch-1 mat-vec whose Q8_1 row is rmsnorm(x_in + delta) * norm_w (the
// decode step's RMSNorm fused into the team kernel; block 0 writes x_in +
// delta to x_out).  Applies to the team kernel with k = 4096 or 8192 and
// 16-byte aligned vectors; qmv_norm_applies says whether it does.
bool qmv_norm_applies(int type, const void* w, int rows, int k, const float* x_in, const float* x_out) {
    int sms = 0;
    if (require_sm100(nullptr, &sms) || !known_type(type) || (k != 4096 && k != 8192) || rows <= 0) return false;
    if (reinterpret_cast<uintptr_t>(x_in) % 16 || reinterpret_cast<uintptr_t>(x_out) % 16 || x_in == x_out) return false;
    TeamPlan plan;
    return plan_team(type, w, x_in, rows, k, 1, sms, plan);
}

p100_status run_qmv_norm(int type, const void* w, int rows, int k, const float* x_in, const float* delta, float* x_out,
                         const float* norm_w, float eps, float* y, unsigned flags, cudaStream_t stream) {
    int sms = 0;
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    TeamPlan plan;
    if (!qmv_norm_applies(type, w, rows, k, x_in, x_out) || !plan_team(type, w, x_in, rows, k, 1, sms, plan) ||
        reinterpret_cast<uintptr_t>(delta) % 16 || reinterpret_cast<uintptr_t>(norm_w) % 16)
        return set_error(P100_ERR_INVALID, "fused RMSNorm mat-vec needs the team kernel with k 4096 or 8192");
    plan.p.w = static_cast<const uint8_t*>(w);
    plan.p.xq = nullptr;
    plan.p.y = y;
    plan.p.col0 = 0;
    plan.p.x_in = x_in;
    plan.p.delta = delta;
    plan.p.x_out = x_out;
    plan.p.norm_w = norm_w;
    plan.p.eps = eps;
    const bool pdl = (flags & P100_QMV_PDL) != 0;
    switch (type) {
        case P100_Q4_0: return launch_team_type<P100_Q4_0>(plan, 1, pdl, stream);
        case P100_Q8_0: return launch_team_type<P100_Q8_0>(plan, 1, pdl, stream);
        case P100_Q4_K: return launch_team_type<P100_Q4_K>(plan, 1, pdl, stream);
        case P100_Q5_K: return launch_team_type<P100_Q5_K>(plan, 1, pdl, stream);
        default: return launch_team_type<P100_Q6_K>(plan, 1, pdl, stream);
    }
}

// ------------------------------------------------------------------ attention
const char* attn_reason(const p100_attn_desc& d) {
    // attention_reference.cpp:18-32, same wording and order.
    if (d.batch <= 0 || d.n_head_q <= 0 || d.n_head_kv <= 0 || d.seq_q <= 0 || d.seq_kv <= 0 || d.d_qk <= 0 ||
        d.d_v <= 0)
        return "all dimensions must be positive";
    if (d.n_head_q % d.n_head_kv != 0) return "n_head_q must be divisible by n_head_kv";
    if (d.softcap < 0.0f || !std::isfinite(d.softcap)) return "softcap must be finite and non-negative";
    if (!std::isfinite(d.scale)) return "scale must be finite";
    return nullptr;
}

constexpr int kFaWideSeq = 8192;
// ... and at least this many (sequence, kv head) pairs: with fewer, one
// 16-CTA cluster per head (cluster merge) beats one part per SM merged
// through the workspace by the last CTA, at any context length.
constexpr int kFaWideHeads = 8;

struct FaPlan {
    int D = 0, G = 0, gmax = 0, parts = 1, nstage = 0;
    long long head_stride = 0, batch_stride = 0;
    size_t smem = 0, ws_o = 0, ws_ml = 0, ws_tickets = 0, ws_total = 0;
    bool auto_parts = false;   // kv_splits == 0: the split may change (fa_mma cluster merge)
    int parts_wide = 1;        // fa_mma with the workspace merge: two CTAs per SM
    int seq = 0;
    int kv_type = P100_KV_F16;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

p100_status plan_fa(const p100_attn_desc& d, int sms, FaPlan& plan) {
    if (const char* why = attn_reason(d)) return set_error(P100_ERR_INVALID, "%s", why);
    if (d.seq_q != 1) return set_error(P100_ERR_UNSUPPORTED, "decode kernel handles seq_q == 1 only");
    if (d.d_qk != d.d_v || (d.d_qk != 64 && d.d_qk != 128 && d.d_qk != 256))
        return set_error(P100_ERR_UNSUPPORTED, "d_qk == d_v in {64, 128, 256} required");
    const int G = d.n_head_q / d.n_head_kv;
    if (G > 8) return set_error(P100_ERR_UNSUPPORTED, "GQA group of %d query heads exceeds 8", G);
    plan.D = d.d_qk;
    plan.G = G;
    plan.gmax = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
    plan.head_stride = d.kv_head_stride ? d.kv_head_stride : static_cast<long long>(d.seq_kv) * d.d_qk;
    plan.batch_stride = d.kv_batch_stride ? d.kv_batch_stride : plan.head_stride * d.n_head_kv;
    if (plan.head_stride < static_cast<long long>(d.seq_kv) * d.d_qk || plan.head_stride % 8 ||
        plan.batch_stride % 8)
        return set_error(P100_ERR_INVALID, "KV strides must cover seq_kv rows and be multiples of 8 elements");
    if (d.kv_type != P100_KV_F16 && d.kv_type != P100_KV_Q8_0 && d.kv_type != P100_KV_Q4_0)
        return set_error(P100_ERR_INVALID, "unknown kv_type %d", d.kv_type);
    plan.kv_type = d.kv_type;
    if (d.kv_type != P100_KV_F16) {
        // fa_mma_kernel only: whole 64-value block pairs keep every row 4-byte aligned
        if (plan.head_stride % 64 || plan.batch_stride % 64)
            return set_error(P100_ERR_INVALID, "quantised KV strides must be multiples of 64 values");
        if ((plan.D != 64 && plan.D != 128) || (G != 1 && G != 2 && G != 4 && G != 8))
            return set_error(P100_ERR_UNSUPPORTED, "quantised K/V need d 64 or 128 and 1, 2, 4 or 8 query heads per kv head");
    }
    const int heads = d.batch * d.n_head_kv;
    const int max_parts = std::max(1, d.seq_kv / fa::kTile);
    int parts = d.kv_splits;
    plan.auto_parts = parts <= 0;
    if (parts <= 0) parts = std::max(1, sms / heads);
    // at most 512 parts: the last-CTA merge keeps every part's (m, l) and
    // weight in shared memory (2 * parts * G floats, inside the idle ring)
    plan.parts = std::min(std::min(parts, max_parts), 512);
    // The 4-warp fa_mma_kernel fits two CTAs per SM (three over a quantised
    // cache: its rings hold raw blocks): with automatic splitting and the
    // workspace merge it runs that many times the parts (the workspace covers
    // both); the 8-warp shape runs plan.parts, one CTA per SM.
    const int per_sm = d.kv_type == P100_KV_Q8_0 || d.kv_type == P100_KV_Q4_0 ? fam::kQuantCtasPerSm : 2;
    plan.parts_wide =
        plan.auto_parts ? std::min(std::min(per_sm * std::max(1, sms / heads), max_parts), 512) : plan.parts;
    plan.seq = d.seq_kv;
    const int ws_parts = std::max(plan.parts, plan.parts_wide);
    plan.nstage = d.d_qk == 256 ? 2 : 4;
    const size_t head = ((64 + (plan.gmax * fa::kTile + fa::kTile * 8 + 24 + plan.gmax * plan.D + 4) * 4) + 127) & ~size_t(127);
    plan.smem = head + size_t(plan.nstage) * 2 * fa::kTile * plan.D * 2;
    if (ws_parts > 1) {
        plan.ws_o = align256(size_t(heads) * ws_parts * G * plan.D * 4);
        plan.ws_ml = align256(size_t(heads) * ws_parts * G * 2 * 4);
        plan.ws_tickets = align256(size_t(heads) * 4);
    }
    plan.ws_total = plan.ws_o + plan.ws_ml + plan.ws_tickets;
    return P100_OK;
}

template <int D, int GMAX>
p100_status launch_fa_t(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t stream, bool pdl) {
    auto kern = fa::fa_decode_kernel<D, GMAX>;
    static thread_local int configured_smem[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_smem[dev] < int(plan.smem)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(plan.smem));
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(fa)");
        configured_smem[dev] = int(plan.smem);
    }
    if (!pdl) {
        kern<<<dim3(plan.parts, heads), fa::kThreads, plan.smem, stream>>>(prm);
        return launch_status("fa_decode_kernel launch");
    }
    // PDL only with a device-resident length: the kernel then waits for the
    // previous kernel before it reads any K/V (see fa::Params::len_dev).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.parts, heads);
    cfg.blockDim = dim3(fa::kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, prm), "fa_decode_kernel launch");
}

// cuTensorMapEncodeTiled from the driver the runtime loaded (no link to libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            f = nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// The fp16 K or V cache as a 4-d tensor (d, rows [0, seq), kv heads, batch)
// in boxes of 64 values x `rows` rows with the 128-byte swizzle.
p100_status kv_tensor_map(CUtensorMap* map, const void* base, int d, int seq, int nkv, int batch,
                          long long head_stride, long long batch_stride, int rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(P100_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[4] = {cuuint64_t(d), cuuint64_t(seq), cuuint64_t(nkv), cuuint64_t(batch)};
    const cuuint64_t strides[3] = {cuuint64_t(d) * 2, cuuint64_t(head_stride) * 2, cuuint64_t(batch_stride) * 2};
    const cuuint32_t box[4] = {64, cuuint32_t(rows), 1, 1};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, elem,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(P100_ERR_INVALID, "K/V tensor map rejected (error %d): strides or extents", int(r));
    return P100_OK;
}

template <int D, int G, int KV, int NW>
p100_status launch_fa_mma_t(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t stream, bool pdl) {
    auto kern = fam::fa_mma_kernel<D, G, KV, NW>;
    constexpr size_t smem = fam::smem_bytes<D, G, KV, NW>();
    static thread_local int configured[64] = {};
    static thread_local int cluster_fits[64][5] = {};   // per log2(parts): clusters that fit, 0 unknown, -1 none
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(fa_mma)");
        configured[dev] = 1;
    }
    // Cluster merge: with automatic splitting and up to 16384 keys, the
    // parts of a kv head become one cluster of np = a power of two <= 16
    // CTAs (and <= G*D/32, so each CTA merges whole Q8_1 blocks), if that
    // keeps at least half the parts.  Longer contexts amortise the workspace
    // merge and run twice the parts instead (two CTAs per SM).
    fa::Params run = prm;
    if (KV == P100_KV_F16) {
        const int batch = heads / prm.nkv;
        if (p100_status st = kv_tensor_map(&run.tmk, prm.k, D, prm.seq, prm.nkv, batch, prm.head_stride,
                                           prm.batch_stride, fam::tile_keys<NW>()))
            return st;
        if (p100_status st = kv_tensor_map(&run.tmv, prm.v, D, prm.seq, prm.nkv, batch, prm.head_stride,
                                           prm.batch_stride, fam::tile_keys<NW>()))
            return st;
    }
    int np = 0;
    if (NW == 4 && plan.auto_parts && plan.parts >= 2 && (plan.seq <= kFaWideSeq || heads < kFaWideHeads)) {
        np = 1;
        while (np * 2 <= std::min(16, plan.parts) && np * 2 <= G * D / 32) np *= 2;
        // A full 16-CTA cluster stays on the cluster merge however many parts
        // the SM count would allow (few kv heads: one cluster per head beats
        // a wide split merged through the workspace by the last CTA).
        if (np < 2 || (2 * np < plan.parts && np < 16)) np = 0;
    }
    int lg = 0;
    while (np && (1 << lg) < np) ++lg;
    if (np && cluster_fits[dev][lg] == 0) {
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(np, 1);
        q.blockDim = dim3(NW * 32);
        q.dynamicSmemBytes = smem;
        cudaLaunchAttribute ca[1];
        ca[0].id = cudaLaunchAttributeClusterDimension;
        ca[0].val.clusterDim.x = np;
        ca[0].val.clusterDim.y = 1;
        ca[0].val.clusterDim.z = 1;
        q.attrs = ca;
        q.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
        cluster_fits[dev][lg] = n >= 1 ? n : -1;
    }
    // every cluster of the launch resident at once, or the GPU full
    if (np && (cluster_fits[dev][lg] < 0 || (cluster_fits[dev][lg] < heads && cluster_fits[dev][lg] * np * 2 < sms_of(dev))))
        np = 0;
    if (np) {
        run.parts = np;
        run.cluster_merge = 1;
    } else if (run.parts > 1 && NW == 4) {
        run.parts = plan.parts_wide;   // the 8-warp shape keeps plan.parts: one CTA per SM
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(run.parts, heads);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (np) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = np;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, run), "fa_mma_kernel launch");
}

template <int D, int KV, int NW>
p100_status launch_fa_mma_nw(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t s, bool pdl) {
    switch (plan.G) {
        case 1: return launch_fa_mma_t<D, 1, KV, NW>(plan, prm, heads, s, pdl);
        case 2: return launch_fa_mma_t<D, 2, KV, NW>(plan, prm, heads, s, pdl);
        case 4: return launch_fa_mma_t<D, 4, KV, NW>(plan, prm, heads, s, pdl);
        default: return launch_fa_mma_t<D, 8, KV, NW>(plan, prm, heads, s, pdl);
    }
}
// The 8-warp shape for automatic splits of more than kFaWideSeq keys over
// at least kFaWideHeads heads (their measured crossover lies between 4K and
// 16K keys), the 4-warp shape else.
template <int D, int KV>
p100_status launch_fa_mma_kv(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t s, bool pdl) {
    if (plan.auto_parts && plan.seq > kFaWideSeq && heads >= kFaWideHeads)
        return launch_fa_mma_nw<D, KV, 8>(plan, prm, heads, s, pdl);
    return launch_fa_mma_nw<D, KV, 4>(plan, prm, heads, s, pdl);
}
template <int D>
p100_status launch_fa_mma_d(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t s, bool pdl) {
    switch (plan.kv_type) {
        case P100_KV_Q8_0: return launch_fa_mma_kv<D, P100_KV_Q8_0>(plan, prm, heads, s, pdl);
        case P100_KV_Q4_0: return launch_fa_mma_kv<D, P100_KV_Q4_0>(plan, prm, heads, s, pdl);
        default: return launch_fa_mma_kv<D, P100_KV_F16>(plan, prm, heads, s, pdl);
    }
}

// The tensor-core kernel serves head_dim 64/128 with 1, 2, 4 or 8 query heads
// per kv head and 16-byte aligned K/V; the SIMT kernel serves the rest.
bool fa_use_mma(const FaPlan& plan, const fa::Params& prm) {
    const bool g_ok = plan.G == 1 || plan.G == 2 || plan.G == 4 || plan.G == 8;
    const bool aligned = reinterpret_cast<uintptr_t>(prm.k) % 16 == 0 && reinterpret_cast<uintptr_t>(prm.v) % 16 == 0;
    return (plan.D == 64 || plan.D == 128) && g_ok && aligned;
}

template <int D>
p100_status launch_fa_d(const FaPlan& plan, const fa::Params& prm, int heads, cudaStream_t s, bool pdl = false) {
    if constexpr (D != 256)
        if (fa_use_mma(plan, prm)) return launch_fa_mma_d<D>(plan, prm, heads, s, pdl);
    if (plan.kv_type != P100_KV_F16)
        return set_error(P100_ERR_UNSUPPORTED, "quantised K/V need the tensor-core kernel (16-byte aligned K/V)");
    switch (plan.gmax) {
        case 1: return launch_fa_t<D, 1>(plan, prm, heads, s, pdl);
        case 2: return launch_fa_t<D, 2>(plan, prm, heads, s, pdl);
        case 4: return launch_fa_t<D, 4>(plan, prm, heads, s, pdl);
        default: return launch_fa_t<D, 8>(plan, prm, heads, s, pdl);
    }
}

}  // namespace
}  // namespace p100b

using namespace p100b;

extern "C" {

int p100_abi_version(void) { return P100_B200_ABI_VERSION; }

const char* p100_last_error(void) { return t_error.c_str(); }

const char* p100_status_name(p100_status s) {
    switch (s) {
        case P100_OK: return "P100_OK";
        case P100_ERR_INVALID: return "P100_ERR_INVALID";
        case P100_ERR_CUDA: return "P100_ERR_CUDA";
        case P100_ERR_NCCL: return "P100_ERR_NCCL";
        case P100_ERR_TIMEOUT: return "P100_ERR_TIMEOUT";
        case P100_ERR_UNSUPPORTED: return "P100_ERR_UNSUPPORTED";
    }
    return "P100_ERR_UNKNOWN";
}

p100_status p100_device_check(int device) {
    clear_error();
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) {
        (void)cudaGetLastError();
        return set_error(P100_ERR_UNSUPPORTED, "no CUDA device");
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        (void)cudaGetLastError();
        return set_error(P100_ERR_UNSUPPORTED, "no CUDA device %d", device);
    }
    p100_status st = require_sm100(nullptr, nullptr);
    cudaSetDevice(cur);
    return st;
}

p100_status p100_device_error(int clear) {
    clear_error();
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    int value = 0;
    if (p100_status st = cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return st;
    if (p100_status st = cuda_status(cudaMemcpyFromSymbol(&value, g_device_error, sizeof value), "read device flag"))
        return st;
    if (clear && value) {
        const int zero = 0;
        if (p100_status st = cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero), "clear device flag"))
            return st;
    }
    if (value == kDevErrInput)
        return set_error(P100_ERR_INVALID, "a kernel read a device-resident token or position out of range");
    return value ? set_error(P100_ERR_TIMEOUT, "a kernel gave up a bounded wait") : P100_OK;
}

int p100_block_elems(int type) { return known_type(type) ? elems_of(type) : -1; }
int p100_block_bytes(int type) { return known_type(type) ? bytes_of(type) : -1; }

size_t p100_weight_bytes(int type, int rows, int k) {
    if (!known_type(type) || rows < 0 || k <= 0 || k % elems_of(type)) return 0;
    return size_t(rows) * (k / elems_of(type)) * bytes_of(type);
}

size_t p100_q8_1_bytes(int k, int batch) {
    if (k <= 0 || k % 32 || batch <= 0) return 0;
    return size_t(batch) * (k / 32) * 36;
}

p100_status p100_q8_1_quantize(const float* x, void* x_q8_1, int k, int batch, p100_stream_t stream) {
    return p100_q8_1_quantize_ex(x, x_q8_1, k, batch, 0u, stream);
}

p100_status p100_q8_1_quantize_ex(const float* x, void* x_q8_1, int k, int batch, unsigned flags,
                                  p100_stream_t stream) {
    clear_error();
    if (flags & ~P100_QMV_PDL) return set_error(P100_ERR_INVALID, "unknown flags 0x%x", flags);
    if (k <= 0 || k % 32) return set_error(P100_ERR_INVALID, "whole activation blocks required");
    if (batch <= 0 || batch > 65535) return set_error(P100_ERR_INVALID, "batch must be in 1..65535");
    if (!x || !x_q8_1) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(x_q8_1) % 4) return set_error(P100_ERR_INVALID, "x_q8_1 must be 4-byte aligned");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    const int blocks = k / 32;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((blocks + 7) / 8, batch);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (flags & P100_QMV_PDL) ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, q8_1_quantize_kernel, x, static_cast<uint8_t*>(x_q8_1), k, blocks),
                       "q8_1_quantize_kernel launch");
}

p100_status p100_dequantize(int type, const void* w, int rows, int k, float* out, p100_stream_t stream) {
    clear_error();
    if (!known_type(type)) return set_error(P100_ERR_INVALID, "unknown weight type %d", type);
    if (k <= 0 || k % elems_of(type)) return set_error(P100_ERR_INVALID, "whole weight blocks required");
    if (rows < 0) return set_error(P100_ERR_INVALID, "rows must be non-negative");
    if (rows == 0) return P100_OK;
    if (!w || !out) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(out) % 16) return set_error(P100_ERR_INVALID, "out must be 16-byte aligned");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    const long long slabs = static_cast<long long>(rows) * (k / 32);
    const dim3 grid(static_cast<unsigned>((slabs + 255) / 256));
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    switch (type) {
        case P100_Q4_0: dequantize_kernel<P100_Q4_0><<<grid, 256, 0, stream>>>(wb, out, rows, k, row_bytes); break;
        case P100_Q8_0: dequantize_kernel<P100_Q8_0><<<grid, 256, 0, stream>>>(wb, out, rows, k, row_bytes); break;
        case P100_Q4_K: dequantize_kernel<P100_Q4_K><<<grid, 256, 0, stream>>>(wb, out, rows, k, row_bytes); break;
        case P100_Q5_K: dequantize_kernel<P100_Q5_K><<<grid, 256, 0, stream>>>(wb, out, rows, k, row_bytes); break;
        default: dequantize_kernel<P100_Q6_K><<<grid, 256, 0, stream>>>(wb, out, rows, k, row_bytes); break;
    }
    return launch_status("dequantize_kernel launch");
}

p100_status p100_kv_to_f16(int kv_type, const void* src, long long ne00, long long ne01, long long ne02,
                           long long ne03, long long s01, long long s02, long long s03, void* dst,
                           p100_stream_t stream) {
    clear_error();
    if (kv_type != P100_KV_Q8_0 && kv_type != P100_KV_Q4_0)
        return set_error(P100_ERR_INVALID, "kv_type must be q8_0 or q4_0, got %d", kv_type);
    if (ne00 <= 0 || ne00 % 32 || ne00 > (1 << 30)) return set_error(P100_ERR_INVALID, "ne00 must be a positive multiple of 32");
    if (ne01 < 0 || ne02 < 0 || ne03 < 0 || s01 < 0 || s02 < 0 || s03 < 0)
        return set_error(P100_ERR_INVALID, "extents and strides must be non-negative");
    if (ne01 * (ne00 / 8) >= (1ll << 31)) return set_error(P100_ERR_INVALID, "ne01 * ne00 / 8 must be below 2^31");
    if (ne01 == 0 || ne02 == 0 || ne03 == 0) return P100_OK;
    if (!src || !dst) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(src) % 2) return set_error(P100_ERR_INVALID, "src must be 2-byte aligned");
    if (reinterpret_cast<uintptr_t>(dst) % 16) return set_error(P100_ERR_INVALID, "dst must be 16-byte aligned");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    kvq::ConvParams p{};
    p.src = static_cast<const uint8_t*>(src);
    p.dst = static_cast<__half*>(dst);
    p.ne01 = ne01;
    p.ne02 = ne02;
    p.ne03 = ne03;
    p.s01 = s01;
    p.s02 = s02;
    p.s03 = s03;
    p.ne00 = static_cast<int>(ne00);
    p.chunks = static_cast<int>(ne00 / 8);
    p.units = static_cast<int>(ne01 * p.chunks);
    const dim3 grid(static_cast<unsigned>((p.units + 256 * kvq::kUnits - 1) / (256 * kvq::kUnits)),
                    static_cast<unsigned>(std::min<long long>(ne02 * ne03, 65535)));
    if (kv_type == P100_KV_Q8_0)
        kvq::kv_to_f16_kernel<P100_KV_Q8_0><<<grid, 256, 0, stream>>>(p);
    else
        kvq::kv_to_f16_kernel<P100_KV_Q4_0><<<grid, 256, 0, stream>>>(p);
    return launch_status("kv_to_f16_kernel launch");
}

p100_status p100_qmv(int type, const void* w, int rows, int k, const void* x_q8_1, int batch, float* y,
                     p100_stream_t stream) {
    clear_error();
    return run_qmv(type, w, rows, k, x_q8_1, batch, y, 0u, stream);
}

p100_status p100_qmv_f32(int type, const void* w, int rows, int k, const float* x, int batch, void* x_q8_1,
                         float* y, unsigned flags, p100_stream_t stream) {
    clear_error();
    if (flags & ~P100_QMV_PDL) return set_error(P100_ERR_INVALID, "unknown flags 0x%x", flags);
    if (!known_type(type)) return set_error(P100_ERR_INVALID, "unknown weight type %d", type);
    if (k <= 0 || k % elems_of(type)) return set_error(P100_ERR_INVALID, "whole weight blocks required");
    if (rows < 0) return set_error(P100_ERR_INVALID, "rows must be non-negative");
    if (batch < 1 || batch > 16) return set_error(P100_ERR_INVALID, "batch must be in 1..16");
    if (rows == 0) return P100_OK;
    if (!w || !x || !y) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(w) % 2) return set_error(P100_ERR_INVALID, "weights must be 2-byte aligned");
    int sms = 0;
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    TeamPlan plan;
    if (!x_q8_1 && plan_team(type, w, x, rows, k, batch, sms, plan)) {
        plan.p.w = static_cast<const uint8_t*>(w);
        plan.p.xq = nullptr;
        plan.p.y = y;
        plan.p.col0 = 0;
        plan.p.x_f32 = x;
        const bool pdl = (flags & P100_QMV_PDL) != 0;
        switch (type) {
            case P100_Q4_0: return launch_team_type<P100_Q4_0>(plan, 1, pdl, stream);
            case P100_Q8_0: return launch_team_type<P100_Q8_0>(plan, 1, pdl, stream);
            case P100_Q4_K: return launch_team_type<P100_Q4_K>(plan, 1, pdl, stream);
            case P100_Q5_K: return launch_team_type<P100_Q5_K>(plan, 1, pdl, stream);
            default: return launch_team_type<P100_Q6_K>(plan, 1, pdl, stream);
        }
    }
    if (!x_q8_1)
        return set_error(P100_ERR_UNSUPPORTED,
                         "without x_q8_1 the quantisation is fused, which needs batch 1 on the team kernel "
                         "(16-byte aligned w and x, rows of whole 16-byte units)");
    if (p100_status st = p100_q8_1_quantize_ex(x, x_q8_1, k, batch, flags, stream)) return st;
    return run_qmv(type, w, rows, k, x_q8_1, batch, y, flags | P100_QMV_PDL, stream);
}

p100_status p100_qmv_ex(int type, const void* w, int rows, int k, const void* x_q8_1, int batch, float* y,
                        unsigned flags, p100_stream_t stream) {
    clear_error();
    if (flags & ~(P100_QMV_PDL | P100_QMV_TC | P100_QMV_MMA))
        return set_error(P100_ERR_INVALID, "unknown flags 0x%x", flags);
    if ((flags & P100_QMV_TC) && (flags & P100_QMV_MMA))
        return set_error(P100_ERR_INVALID, "P100_QMV_TC and P100_QMV_MMA exclude each other");
    return run_qmv(type, w, rows, k, x_q8_1, batch, y, flags, stream);
}

p100_status p100_attn_validate(const p100_attn_desc* desc, char* why, size_t why_len) {
    clear_error();
    if (!desc) return set_error(P100_ERR_INVALID, "null descriptor");
    const char* reason = attn_reason(*desc);
    if (why && why_len) std::snprintf(why, why_len, "%s", reason ? reason : "");
    return reason ? set_error(P100_ERR_INVALID, "%s", reason) : P100_OK;
}

size_t p100_fa_workspace_size(const p100_attn_desc* desc) {
    clear_error();
    if (!desc) return 0;
    if (const char* why = attn_reason(*desc)) {
        set_error(P100_ERR_INVALID, "%s", why);
        return 0;
    }
    int sms = 0;
    if (require_sm100(nullptr, &sms)) return 0;
    FaPlan plan;
    if (plan_fa(*desc, sms, plan)) return 0;
    return plan.ws_total;
}

p100_status p100_fa_workspace_init(void* ws, size_t ws_bytes, p100_stream_t stream) {
    clear_error();
    if (!ws || !ws_bytes) return P100_OK;
    return cuda_status(cudaMemsetAsync(ws, 0, ws_bytes, stream), "cudaMemsetAsync(workspace)");
}

p100_status p100_fa_decode(const p100_attn_desc* desc, const float* q, const void* k, const void* v,
                           const float* mask, float* o, float* lse, void* ws, size_t ws_bytes,
                           p100_stream_t stream) {
    clear_error();
    if (!desc) return set_error(P100_ERR_INVALID, "null descriptor");
    int sms = 0;
    if (const char* why = attn_reason(*desc)) return set_error(P100_ERR_INVALID, "%s", why);
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    FaPlan plan;
    if (p100_status st = plan_fa(*desc, sms, plan)) return st;
    if (!q || !k || !v || !o) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16)
        return set_error(P100_ERR_INVALID, "K and V must be 16-byte aligned");
    if (plan.ws_total > ws_bytes || (plan.ws_total && !ws))
        return set_error(P100_ERR_INVALID, "workspace of %zu bytes needed, %zu given", plan.ws_total, ws_bytes);
    if (reinterpret_cast<uintptr_t>(ws) % 256) return set_error(P100_ERR_INVALID, "workspace must be 256-byte aligned");
    fa::Params prm = {};
    prm.q = q;
    prm.k = static_cast<const __half*>(k);
    prm.v = static_cast<const __half*>(v);
    prm.mask = mask;
    prm.o = o;
    prm.lse = lse;
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    prm.ws_o = plan.parts > 1 ? reinterpret_cast<float*>(wsb) : nullptr;
    prm.ws_ml = plan.parts > 1 ? reinterpret_cast<float*>(wsb + plan.ws_o) : nullptr;
    prm.tickets = plan.parts > 1 ? reinterpret_cast<unsigned*>(wsb + plan.ws_o + plan.ws_ml) : nullptr;
    prm.nkv = desc->n_head_kv;
    prm.G = plan.G;
    prm.seq = desc->seq_kv;
    prm.parts = plan.parts;
    prm.nstage = plan.nstage;
    prm.head_stride = plan.head_stride;
    prm.batch_stride = plan.batch_stride;
    prm.scale = desc->scale == 0.0f ? 1.0f / std::sqrt(static_cast<float>(desc->d_qk)) : desc->scale;
    prm.softcap = desc->softcap;
    const int heads = desc->batch * desc->n_head_kv;
    switch (plan.D) {
        case 64: return launch_fa_d<64>(plan, prm, heads, stream);
        case 128: return launch_fa_d<128>(plan, prm, heads, stream);
        default: return launch_fa_d<256>(plan, prm, heads, stream);
    }
}

}  // extern "C"

// ------------------------------------------------------------------ h16 path
namespace p100b {
namespace {
template <int TYPE, int CHAIN>
p100_status launch_h16_t(const h16::Params& p, int grid, cudaStream_t stream) {
    h16::qmv_h16_kernel<TYPE, CHAIN><<<grid, h16::kThreads, h16::kWarps * sizeof(float), stream>>>(p);
    return launch_status("qmv_h16_kernel launch");
}
template <int TYPE>
p100_status launch_h16_type(const h16::Params& p, int chain, int grid, cudaStream_t s) {
    return chain == 8 ? launch_h16_t<TYPE, 8>(p, grid, s) : launch_h16_t<TYPE, 16>(p, grid, s);
}
}  // namespace
}  // namespace p100b

extern "C" p100_status p100_h16_prepare(const float* x, void* h, float* ss, int k, int batch, p100_stream_t stream) {
    clear_error();
    if (k <= 0 || k % 32) return set_error(P100_ERR_INVALID, "whole activation blocks required");
    if (batch <= 0) return set_error(P100_ERR_INVALID, "batch must be positive");
    if (!x || !h || !ss) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(ss) % 8) return set_error(P100_ERR_INVALID, "ss must be 8-byte aligned");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    const long long nblk = static_cast<long long>(batch) * (k / 32);
    if (nblk > (1ll << 30)) return set_error(P100_ERR_INVALID, "activation too large");
    const int per = 256 / 32;
    h16::h16_prepare_kernel<<<static_cast<int>((nblk + per - 1) / per), 256, 0, stream>>>(
        x, static_cast<__half*>(h), reinterpret_cast<float2*>(ss), k, static_cast<int>(nblk));
    return launch_status("h16_prepare_kernel launch");
}

extern "C" p100_status p100_qmv_h16(int type, const void* w, int rows, int k, const void* h, const float* ss, int batch,
                                    int chain, float* y, p100_stream_t stream) {
    clear_error();
    if (!known_type(type)) return set_error(P100_ERR_INVALID, "unknown weight type %d", type);
    if (!ref_type(type)) return set_error(P100_ERR_UNSUPPORTED, "the h16 path covers Q4_0, Q8_0 and Q4_K");
    if (k <= 0 || k % elems_of(type)) return set_error(P100_ERR_INVALID, "whole weight blocks required");
    if (chain != 8 && chain != 16) return set_error(P100_ERR_INVALID, "invalid h16 shape/chain");
    if (rows < 0 || batch <= 0) return set_error(P100_ERR_INVALID, "rows must be non-negative and batch positive");
    if (!w || !h || !ss || !y) return set_error(P100_ERR_INVALID, "null buffer");
    if (k % h16::kLaneElems || k / h16::kLaneElems > h16::kThreads)
        return set_error(P100_ERR_UNSUPPORTED, "h16 mat-vec needs k a multiple of 128, at most %d",
                         h16::kLaneElems * h16::kThreads);
    if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(h) % 16 ||
        reinterpret_cast<uintptr_t>(ss) % 8)
        return set_error(P100_ERR_INVALID, "w and h must be 16-byte aligned, ss 8-byte aligned");
    int sms = 0;
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    if (rows == 0) return P100_OK;
    h16::Params p{};
    p.w = static_cast<const uint8_t*>(w);
    p.rows = rows;
    p.k = k;
    p.row_bytes = static_cast<int>(size_t(k / elems_of(type)) * bytes_of(type));
    p.team = k / h16::kLaneElems;
    int pad = 1;
    while (pad < p.team) pad *= 2;
    p.team_pad = pad;
    const int teams = h16::kThreads / pad;
    const int grid = std::max(1, std::min(sms, (rows + teams - 1) / teams));
    for (int c = 0; c < batch; ++c) {
        p.h = static_cast<const __half*>(h) + size_t(c) * k;
        p.ss = reinterpret_cast<const float2*>(ss) + size_t(c) * (k / 32);
        p.y = y + size_t(c) * rows;
        p100_status st;
        switch (type) {
            case P100_Q4_0: st = launch_h16_type<P100_Q4_0>(p, chain, grid, stream); break;
            case P100_Q8_0: st = launch_h16_type<P100_Q8_0>(p, chain, grid, stream); break;
            default: st = launch_h16_type<P100_Q4_K>(p, chain, grid, stream); break;
        }
        if (st) return st;
    }
    return P100_OK;
}

// ------------------------------------------------------------------ decode without a workspace argument
// For callers that may not allocate device memory (see p100_fa_decode_static
// in p100/b200.h): the split-K partials go to one fixed array per device
// instead of a caller-owned workspace.  The array is part of this library's
// device module, so every GPU that loads the library holds it until exit.
namespace p100b {
static __device__ __align__(256) unsigned char g_fa_static_scratch[P100_FA_STATIC_SCRATCH_BYTES];
namespace {
std::mutex g_static_mutex;
// The array's device address per device ordinal, valid for the context whose
// unique id is beside it: a cudaDeviceReset or a recreated primary context
// gets a new id, and the address is looked up again.
void* g_static_scratch_ptr[64];
unsigned long long g_static_scratch_ctx[64];

// Unique id of the calling thread's current context (0 if unavailable), from
// the driver the runtime loaded.
unsigned long long current_context_id() {
    static const auto fns = [] {
        std::pair<PFN_cuCtxGetCurrent_v4000, PFN_cuCtxGetId_v12000> r{nullptr, nullptr};
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            r.first = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            r.second = reinterpret_cast<PFN_cuCtxGetId_v12000>(f);
        (void)cudaGetLastError();
        return r;
    }();
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!fns.first || !fns.second || fns.first(&ctx) != CUDA_SUCCESS || !ctx || fns.second(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}
}  // namespace
}  // namespace p100b

extern "C" p100_status p100_fa_decode_static(const p100_attn_desc* desc, const float* q, const void* k,
                                             const void* v, const float* mask, float* o, float* lse,
                                             p100_stream_t stream) {
    clear_error();
    if (!desc) return set_error(P100_ERR_INVALID, "null descriptor");
    if (const char* why = attn_reason(*desc)) return set_error(P100_ERR_INVALID, "%s", why);
    int dev = 0, sms = 0;
    if (p100_status st = require_sm100(&dev, &sms)) return st;
    FaPlan plan;
    if (p100_status st = plan_fa(*desc, sms, plan)) return st;
    if (plan.ws_total > P100_FA_STATIC_SCRATCH_BYTES)
        return set_error(P100_ERR_INVALID,
                         "split-K partials need %zu bytes, more than the %u-byte static scratch; lower kv_splits",
                         plan.ws_total, static_cast<unsigned>(P100_FA_STATIC_SCRATCH_BYTES));
    void* scratch = nullptr;
    if (plan.ws_total) {
        {
            // Host code cannot use the array's name as a device address: look
            // the address up once per device and context, with that device
            // current.  The lookup creates the context if there is none yet,
            // so its id is read after it.
            std::lock_guard<std::mutex> lock(g_static_mutex);
            const unsigned long long ctx = current_context_id();
            if (!g_static_scratch_ptr[dev] || ctx == 0 || g_static_scratch_ctx[dev] != ctx) {
                void* ptr = nullptr;
                if (p100_status st = cuda_status(cudaGetSymbolAddress(&ptr, g_fa_static_scratch),
                                                 "cudaGetSymbolAddress(static scratch)"))
                    return st;
                g_static_scratch_ptr[dev] = ptr;
                g_static_scratch_ctx[dev] = current_context_id();
            }
            scratch = g_static_scratch_ptr[dev];
        }
        // The array keeps the previous call's contents; the per-head tickets
        // of the combine must start at zero.
        if (p100_status st = cuda_status(
                cudaMemsetAsync(static_cast<uint8_t*>(scratch) + plan.ws_o + plan.ws_ml, 0, plan.ws_tickets, stream),
                "cudaMemsetAsync(static scratch tickets)"))
            return st;
    }
    return p100_fa_decode(desc, q, k, v, mask, o, lse, scratch, plan.ws_total, stream);
}

// The batch-1 decoder and the decode-step glue entry points.
#include "decoder.cuh"

// ------------------------------------------------ peer all-reduce (tp.cpp)
// The launch behind p100_tp_allreduce_sum's peer path: tp.cpp is host-only
// C++, so it reaches the kernel through this function of plain types.
// slots[r] = rank r's arena of [2][world][n_cap] tagged words (this rank's
// own at slots[rank]); epoch, ticket and broken are this rank's device ints;
// wait_ns bounds each wait for another rank.
namespace p100b {
p100_status peer_allreduce(float* buf, size_t count, unsigned long long* const* slots, int world, int rank, int n_cap,
                           int* epoch, int* ticket, int* broken, unsigned long long wait_ns, cudaStream_t stream) {
    if (world < 1 || world > dec::kArMaxRanks || count > size_t(n_cap) || n_cap % 4)
        return set_error(P100_ERR_INVALID, "peer all-reduce: %zu values, %d ranks, room for %d", count, world, n_cap);
    if (count == 0) return P100_OK;
    dec::PeerAr ar{};
    for (int r = 0; r < world; ++r) ar.slots[r] = slots[r];
    ar.world = world;
    ar.rank = rank;
    ar.n = n_cap;
    ar.epoch = epoch;
    ar.wait_ns = wait_ns;
    // a programmatic dependent of the previous kernel: its launch overlaps
    // that kernel's tail, and it reads nothing before griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((count + 4 * dec::kArThreads - 1) / (4 * dec::kArThreads)));
    cfg.blockDim = dim3(dec::kArThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, dec::peer_allreduce_kernel, buf, static_cast<int>(count), ar, ticket, broken),
                       "peer_allreduce_kernel launch");
}

// Device scratch of the peer path's set-up exchanges in p100_tp_init_rank (a
// gather's input and output and an agreement word).  A static array, so
// every rank has it and enters every collective of the set-up.
static __device__ float g_tp_setup_scratch[16 + 16 * dec::kArMaxRanks + 4];
float* tp_setup_scratch() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tp_setup_scratch) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return static_cast<float*>(p);
}
}  // namespace p100b
