// tp.cpp — tensor-parallel communicator for the row-split decode layout.
//
// The reference moves data between its two GPUs with a peer/staged copy
// layer (src/p2p/p2p.cpp) and exercises llama.cpp's "-sm tensor" NCCL
// all-reduce only from its A/B kit (bench/phase0.sh:154-164).  On one
// 8xB200 box the per-layer exchange of a row-split model is an fp32
// partial-sum all-reduce of the hidden vector, issued here through NCCL over
// NVLink/NVSwitch, one communicator rank per GPU.
//
// All-reduces of up to P100_TP_PEER_MAX values run over NVLink peer memory
// instead of NCCL when every pair of the group's GPUs has peer access (the
// ranks agree while joining; P100_TP_ALLREDUCE=nccl keeps NCCL): one kernel
// pushes each rank's values into every rank's slot arena (CUDA IPC mappings)
// as 64-bit words tagged with the call's epoch and sums them in rank order,
// the decoder's exchange as a plain collective (dec::peer_allreduce_kernel).
// At these sizes NCCL's all-reduce measured about 21 us a call.
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

#include <algorithm>
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
// In capi.cu (the CUDA translation unit).
p100_status peer_allreduce(float* buf, size_t count, unsigned long long* const* slots, int world, int rank, int n_cap,
                           int* epoch, int* ticket, int* broken, unsigned long long wait_ns, cudaStream_t stream);
float* tp_setup_scratch();
}  // namespace p100b

namespace {
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerCap = P100_TP_PEER_MAX;
constexpr size_t kPeerSlotBytes(int world) { return size_t(2) * size_t(world) * kPeerCap * 8; }
// How long a peer all-reduce waits for the other ranks: ranks may reach a
// collective seconds apart (as NCCL allows), so far longer than a kernel's
// own waits; a wait that runs out marks the exchange broken, and later calls
// give up at once.
constexpr unsigned long long kPeerWaitNs = 30ull * 1000 * 1000 * 1000;
}  // namespace

struct p100_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1, device = 0;
    // the peer path (multi-process groups whose GPUs all reach each other)
    bool peer = false;
    unsigned char* arena = nullptr;           // this rank's [2][size][kPeerCap] words, then epoch, ticket, broken
    void* mapped[kPeerMaxRanks] = {};         // the other ranks' arenas (IPC mappings)
    unsigned long long* slots[kPeerMaxRanks] = {};
    int* epoch = nullptr;
    int* ticket = nullptr;
    int* broken = nullptr;
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

// The set-up exchanges of the peer path.  Every rank calls every exchange,
// in the same order, whatever its local state: a local failure is carried
// into the next agreement (an all-reduce of failure counts) instead of
// skipping a collective, so no rank is left waiting in one.
struct PeerSetup {
    p100_tp* tp;
    cudaStream_t s = nullptr;
    float* buf = nullptr;
    p100_status err = P100_OK;   // the first local error of an exchange
    explicit PeerSetup(p100_tp* t) : tp(t) {
        note(cuda_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "peer set-up stream"));
        buf = tp_setup_scratch();
        if (!buf) note(set_error(P100_ERR_CUDA, "peer set-up scratch"));
    }
    ~PeerSetup() {
        if (s) cudaStreamDestroy(s);
    }
    void note(p100_status st) {
        if (st && !err) err = st;
    }
    bool usable() const { return s && buf; }
    // every rank's `count` floats (count <= 16) into out, rank-major
    void gather(const float* mine, int count, float* out) {
        if (!usable()) {
            std::fill(out, out + size_t(count) * tp->size, 0.f);
            return;
        }
        note(cuda_status(cudaMemcpyAsync(buf, mine, sizeof(float) * count, cudaMemcpyHostToDevice, s), "gather in"));
        note(nccl_status(nccl().allGather(buf, buf + 16, size_t(count), ncclFloat32, tp->comm, s), "ncclAllGather"));
        note(cuda_status(cudaMemcpyAsync(out, buf + 16, sizeof(float) * count * tp->size, cudaMemcpyDeviceToHost, s),
                         "gather out"));
        note(cuda_status(cudaStreamSynchronize(s), "gather sync"));
    }
    // Over all ranks: 1000 x (ranks with an exchange error so far) + (ranks
    // that passed ok = false).  Every rank gets the same number.
    int agree(bool ok) {
        const float mine = (err ? 1000.f : 0.f) + (ok ? 0.f : 1.f);
        float all = 1000.f * tp->size;
        if (usable()) {
            float* at = buf + 16 + 16 * kPeerMaxRanks;
            note(cuda_status(cudaMemcpyAsync(at, &mine, sizeof(float), cudaMemcpyHostToDevice, s), "agree in"));
            note(nccl_status(nccl().allReduce(at, at, 1, ncclFloat32, ncclSum, tp->comm, s), "ncclAllReduce"));
            note(cuda_status(cudaMemcpyAsync(&all, at, sizeof(float), cudaMemcpyDeviceToHost, s), "agree out"));
            note(cuda_status(cudaStreamSynchronize(s), "agree sync"));
        }
        return static_cast<int>(all + 0.5f);
    }
    p100_status fail() {
        return err ? err : set_error(P100_ERR_CUDA, "peer all-reduce set-up: another rank failed");
    }
};

void release_peer(p100_tp* tp) {
    for (int r = 0; r < kPeerMaxRanks; ++r)
        if (tp->mapped[r]) {
            cudaIpcCloseMemHandle(tp->mapped[r]);
            tp->mapped[r] = nullptr;
        }
    if (tp->arena) cudaFree(tp->arena);
    tp->arena = nullptr;
    tp->peer = false;
    for (auto& p : tp->slots) p = nullptr;
    tp->epoch = tp->ticket = tp->broken = nullptr;
}

// Collective, right after the group is joined (tp->device current): decides,
// every rank agreeing, whether all-reduces of up to kPeerCap values go over
// peer memory, and maps every rank's slot arena.  A rank that declines (no
// peer access to some rank, P100_TP_ALLREDUCE=nccl, an arena or IPC mapping
// that fails: ranks in one process cannot map each other's arenas) leaves
// every rank on NCCL; only a failure of the set-up's own exchanges is an
// error, on every rank.
p100_status setup_peer(p100_tp* tp) {
    const int world = tp->size;
    if (world < 2 || world > kPeerMaxRanks) return P100_OK;   // the same decision on every rank
    PeerSetup ps(tp);
    // 1. every rank's device -> peer access to all of them
    std::vector<float> devs(size_t(world), 0.f);
    const float me = float(tp->device);
    ps.gather(&me, 1, devs.data());
    const char* mode = std::getenv("P100_TP_ALLREDUCE");
    bool ok = !(mode && std::strcmp(mode, "nccl") == 0);
    for (int r = 0; r < world && ok; ++r) {
        if (r == tp->rank) continue;
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, tp->device, int(devs[size_t(r)])) != cudaSuccess || !can) ok = false;
    }
    (void)cudaGetLastError();
    int v = ps.agree(ok);
    if (v >= 1000) return ps.fail();
    if (v) return P100_OK;
    // 2. this rank's arena and its IPC handle
    const size_t bytes = kPeerSlotBytes(world) + 256;   // slots | epoch, ticket, broken
    cudaIpcMemHandle_t h{};
    ok = cudaMalloc(&tp->arena, bytes) == cudaSuccess;
    if (!ok) tp->arena = nullptr;
    ok = ok && cudaMemset(tp->arena, 0, bytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
         cudaIpcGetMemHandle(&h, tp->arena) == cudaSuccess;
    (void)cudaGetLastError();
    v = ps.agree(ok);
    if (v) {
        release_peer(tp);
        return v >= 1000 ? ps.fail() : P100_OK;
    }
    // 3. every rank's handle; map the others' arenas
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    std::vector<float> hmine(16), hall(size_t(world) * 16);
    std::memcpy(hmine.data(), &h, 64);
    ps.gather(hmine.data(), 16, hall.data());
    for (int r = 0; r < world && ok; ++r) {
        if (r == tp->rank) {
            tp->slots[r] = reinterpret_cast<unsigned long long*>(tp->arena);
            continue;
        }
        cudaIpcMemHandle_t hr;
        std::memcpy(&hr, hall.data() + size_t(r) * 16, 64);
        void* p = nullptr;
        ok = cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        tp->mapped[r] = ok ? p : nullptr;
        tp->slots[r] = static_cast<unsigned long long*>(p);
    }
    (void)cudaGetLastError();
    // 4. every rank's arena is zeroed and mapped before any rank pushes
    v = ps.agree(ok);
    if (v) {
        release_peer(tp);
        return v >= 1000 ? ps.fail() : P100_OK;
    }
    tp->epoch = reinterpret_cast<int*>(tp->arena + kPeerSlotBytes(world));
    tp->ticket = reinterpret_cast<int*>(tp->arena + kPeerSlotBytes(world) + 128);
    tp->broken = reinterpret_cast<int*>(tp->arena + kPeerSlotBytes(world) + 192);
    tp->peer = true;
    return P100_OK;
}
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
    if (p100_status st = setup_peer(tp)) {
        release_peer(tp);
        nccl().commDestroy(tp->comm);
        delete tp;
        return st;
    }
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
int p100_tp_peer(const p100_tp* tp) { return tp && tp->peer ? 1 : 0; }

p100_status p100_tp_allreduce_sum(p100_tp* tp, float* buf, size_t count, p100_stream_t stream) {
    clear_error();
    if (!tp || (!buf && count)) return set_error(P100_ERR_INVALID, "null argument");
    if (count == 0) return P100_OK;
    DeviceScope scope;
    if (p100_status st = cuda_status(cudaSetDevice(tp->device), "cudaSetDevice")) return st;
    // the path depends only on count, which every rank passes the same
    if (tp->peer && count <= size_t(kPeerCap))
        return peer_allreduce(buf, count, tp->slots, tp->size, tp->rank, kPeerCap, tp->epoch, tp->ticket, tp->broken,
                              kPeerWaitNs, stream);
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
    if (tp->arena) {
        cudaDeviceSynchronize();   // no peer all-reduce of this rank still reads or writes the arenas
        release_peer(tp);
    }
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
