// tp.cpp — tensor-parallel communicator for the row-split decode layout.
//
// The reference moves data between its two GPUs with a peer/staged copy
// layer (src/p2p/p2p.cpp) and exercises llama.cpp's "-sm tensor" NCCL
// all-reduce only from its A/B kit (bench/phase0.sh:154-164).  On one
// 8xB200 box the per-layer exchange of a row-split model is an fp32
// partial-sum all-reduce of the hidden vector, issued here through NCCL over
// NVLink/NVSwitch, one communicator rank per GPU.
//
// Failure handling: every NCCL call's status becomes P100_ERR_NCCL with
// ncclGetErrorString text; destroy aborts a communicator that reports an
// asynchronous error instead of waiting on it.  P100_FAULT=tp_init makes
// init fail on the host (for tests of the error path; no GPU involvement).
//
// NCCL is bound at first use with dlopen rather than linked: a process that
// already holds an NCCL (PyTorch loads its own libnccl.so.2) keeps that one,
// so two NCCL builds never meet in one process.  P100_NCCL_LIB names a
// specific library file.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <type_traits>
#include <string>
#include <vector>

#include "p100/b200.h"

namespace p100b {
p100_status set_error(p100_status status, const char* fmt, ...);
p100_status cuda_status(cudaError_t err, const char* what);
void clear_error();
p100_status require_sm100(int* device_out, int* sm_count_out);
bool fault_injected(const char* name);
}  // namespace p100b

struct p100_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1, device = 0;
};

using namespace p100b;

namespace p100b {
// P100_FAULT is a comma-separated list of host-side fault names.
bool fault_injected(const char* name) {
    const char* env = std::getenv("P100_FAULT");
    if (!env || !*env) return false;
    const size_t n = std::strlen(name);
    for (const char* p = env; *p;) {
        const char* end = std::strchr(p, ',');
        const size_t len = end ? size_t(end - p) : std::strlen(p);
        if (len == n && std::strncmp(p, name, n) == 0) return true;
        if (!end) break;
        p = end + 1;
    }
    return false;
}
}  // namespace p100b

namespace {
// The NCCL entry points this layer uses, resolved from one library handle.
struct Nccl {
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRank) commInitRank = nullptr;
    decltype(&ncclCommInitAll) commInitAll = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
    decltype(&ncclAllGather) allGather = nullptr;
    decltype(&ncclGroupStart) groupStart = nullptr;
    decltype(&ncclGroupEnd) groupEnd = nullptr;
    decltype(&ncclCommDestroy) commDestroy = nullptr;
    decltype(&ncclCommAbort) commAbort = nullptr;
    decltype(&ncclCommGetAsyncError) commGetAsyncError = nullptr;
    decltype(&ncclGetErrorString) getErrorString = nullptr;
    std::string error;
};

const Nccl& nccl() {
    static Nccl api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = nullptr;
        if (const char* path = std::getenv("P100_NCCL_LIB")) h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);   // already in the process
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* why = dlerror();
            api.error = std::string("cannot load libnccl.so.2: ") + (why ? why : "unknown");
            return;
        }
        auto bind = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn && api.error.empty()) api.error = std::string("libnccl.so.2 lacks ") + name;
        };
        bind(api.getUniqueId, "ncclGetUniqueId");
        bind(api.commInitRank, "ncclCommInitRank");
        bind(api.commInitAll, "ncclCommInitAll");
        bind(api.allReduce, "ncclAllReduce");
        bind(api.allGather, "ncclAllGather");
        bind(api.groupStart, "ncclGroupStart");
        bind(api.groupEnd, "ncclGroupEnd");
        bind(api.commDestroy, "ncclCommDestroy");
        bind(api.commAbort, "ncclCommAbort");
        bind(api.commGetAsyncError, "ncclCommGetAsyncError");
        bind(api.getErrorString, "ncclGetErrorString");
    });
    return api;
}

p100_status nccl_ready() {
    const Nccl& api = nccl();
    return api.error.empty() ? P100_OK : set_error(P100_ERR_NCCL, "%s", api.error.c_str());
}

p100_status nccl_status(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return P100_OK;
    return set_error(P100_ERR_NCCL, "%s: %s", what, nccl().getErrorString(r));
}

// Restores the caller's current device on scope exit.
struct DeviceScope {
    int saved = -1;
    DeviceScope() {
        if (cudaGetDevice(&saved) != cudaSuccess) {
            (void)cudaGetLastError();
            saved = -1;
        }
    }
    ~DeviceScope() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};
}  // namespace

extern "C" {

p100_status p100_tp_unique_id(void* id) {
    clear_error();
    static_assert(sizeof(ncclUniqueId) == P100_TP_ID_BYTES, "ncclUniqueId size");
    if (!id) return set_error(P100_ERR_INVALID, "null id buffer");
    if (p100_status st = nccl_ready()) return st;
    ncclUniqueId uid;
    if (p100_status st = nccl_status(nccl().getUniqueId(&uid), "ncclGetUniqueId")) return st;
    std::memcpy(id, &uid, sizeof uid);
    return P100_OK;
}

p100_status p100_tp_init_rank(const void* id, int nranks, int rank, int device, p100_tp** out) {
    clear_error();
    if (!id || !out) return set_error(P100_ERR_INVALID, "null argument");
    if (nranks < 1 || rank < 0 || rank >= nranks) return set_error(P100_ERR_INVALID, "rank %d of %d", rank, nranks);
    *out = nullptr;
    if (fault_injected("tp_init")) return set_error(P100_ERR_NCCL, "injected fault: tp_init (P100_FAULT)");
    if (p100_status st = nccl_ready()) return st;
    DeviceScope scope;
    if (p100_status st = cuda_status(cudaSetDevice(device), "cudaSetDevice")) return st;
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    auto* tp = new (std::nothrow) p100_tp;
    if (!tp) return set_error(P100_ERR_INVALID, "out of host memory");
    if (p100_status st = nccl_status(nccl().commInitRank(&tp->comm, nranks, uid, rank), "ncclCommInitRank")) {
        delete tp;
        return st;
    }
    tp->rank = rank;
    tp->size = nranks;
    tp->device = device;
    *out = tp;
    return P100_OK;
}

p100_status p100_tp_create(int ngpu, const int* devs, p100_tp** out) {
    clear_error();
    if (ngpu < 1 || !devs || !out) return set_error(P100_ERR_INVALID, "bad arguments");
    if (fault_injected("tp_init")) return set_error(P100_ERR_NCCL, "injected fault: tp_init (P100_FAULT)");
    if (p100_status st = nccl_ready()) return st;
    DeviceScope scope;
    for (int i = 0; i < ngpu; ++i) {
        if (p100_status st = cuda_status(cudaSetDevice(devs[i]), "cudaSetDevice")) return st;
        if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    }
    std::vector<ncclComm_t> comms(ngpu);
    if (p100_status st = nccl_status(nccl().commInitAll(comms.data(), ngpu, devs), "ncclCommInitAll")) return st;
    for (int i = 0; i < ngpu; ++i) {
        out[i] = new p100_tp;
        out[i]->comm = comms[i];
        out[i]->rank = i;
        out[i]->size = ngpu;
        out[i]->device = devs[i];
    }
    return P100_OK;
}

int p100_tp_rank(const p100_tp* tp) { return tp ? tp->rank : -1; }
int p100_tp_size(const p100_tp* tp) { return tp ? tp->size : -1; }
int p100_tp_device(const p100_tp* tp) { return tp ? tp->device : -1; }

p100_status p100_tp_allreduce_sum(p100_tp* tp, float* buf, size_t count, p100_stream_t stream) {
    clear_error();
    if (!tp || (!buf && count)) return set_error(P100_ERR_INVALID, "null argument");
    if (count == 0) return P100_OK;
    DeviceScope scope;
    if (p100_status st = cuda_status(cudaSetDevice(tp->device), "cudaSetDevice")) return st;
    return nccl_status(nccl().allReduce(buf, buf, count, ncclFloat32, ncclSum, tp->comm, stream), "ncclAllReduce");
}

p100_status p100_tp_allreduce_sum_group(p100_tp* const* tps, int n, float* const* bufs, size_t count,
                                        const p100_stream_t* streams) {
    clear_error();
    if (!tps || !bufs || !streams || n < 1) return set_error(P100_ERR_INVALID, "null argument");
    if (count == 0) return P100_OK;
    DeviceScope scope;
    if (p100_status st = nccl_status(nccl().groupStart(), "ncclGroupStart")) return st;
    p100_status first = P100_OK;
    for (int i = 0; i < n && !first; ++i) {
        first = cuda_status(cudaSetDevice(tps[i]->device), "cudaSetDevice");
        if (!first)
            first = nccl_status(nccl().allReduce(bufs[i], bufs[i], count, ncclFloat32, ncclSum, tps[i]->comm, streams[i]),
                                "ncclAllReduce");
    }
    p100_status end = nccl_status(nccl().groupEnd(), "ncclGroupEnd");
    return first ? first : end;
}

p100_status p100_tp_allgather(p100_tp* tp, const float* in, float* out, size_t count, p100_stream_t stream) {
    clear_error();
    if (!tp || ((!in || !out) && count)) return set_error(P100_ERR_INVALID, "null argument");
    if (count == 0) return P100_OK;
    DeviceScope scope;
    if (p100_status st = cuda_status(cudaSetDevice(tp->device), "cudaSetDevice")) return st;
    return nccl_status(nccl().allGather(in, out, count, ncclFloat32, tp->comm, stream), "ncclAllGather");
}

p100_status p100_tp_destroy(p100_tp* tp) {
    clear_error();
    if (!tp) return P100_OK;
    DeviceScope scope;
    cudaSetDevice(tp->device);
    p100_status st = P100_OK;
    if (tp->comm) {
        ncclResult_t async = ncclSuccess;
        nccl().commGetAsyncError(tp->comm, &async);
        if (async != ncclSuccess) {
            st = nccl_status(async, "communicator async error");
            nccl().commAbort(tp->comm);
        } else {
            st = nccl_status(nccl().commDestroy(tp->comm), "ncclCommDestroy");
        }
    }
    delete tp;
    return st;
}

}  // extern "C"
