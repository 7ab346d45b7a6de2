// p2p.cpp — peer copy layer for one B200 box (interface: include/p100/p2p.h).
//
// Behaviour follows the reference's src/p2p/p2p.cpp contract:
//   * probe/describe report every device and the peer matrix
//     (p2p.cpp:55-108), leaving the caller's device current;
//   * a link uses the Peer path when both directions can be enabled and
//     P100_DISABLE_P2P is unset (p2p.cpp:48-51,148-178), else Staged;
//   * copies are stream-ordered, successive copies on one link are ordered
//     even across streams, and the destructor drains the link's own work
//     before freeing anything (p2p.cpp:110-146,183-222).
// The Staged path stages chunks through two pinned host buffers: device ->
// host on the caller's stream, host -> device on the link's own stream on the
// destination device, with events handing each buffer back and forth.
#include "p100/p2p.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <sstream>
#include <stdexcept>

#include "p100/b200.h"

namespace p100b {
p100_status set_error(p100_status status, const char* fmt, ...);
void clear_error();
}  // namespace p100b

namespace p100::p2p {
namespace {

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

// Remembers the caller's device and puts it back when the scope ends.
class CurrentDevice {
public:
    CurrentDevice() { check(cudaGetDevice(&saved_), "cudaGetDevice"); }
    void use(int dev) { check(cudaSetDevice(dev), "cudaSetDevice"); }
    ~CurrentDevice() {
        if (cudaSetDevice(saved_) != cudaSuccess) (void)cudaGetLastError();
    }
    CurrentDevice(const CurrentDevice&) = delete;
    CurrentDevice& operator=(const CurrentDevice&) = delete;

private:
    int saved_ = 0;
};

// Enables access from `dev` to `peer`; true if access is (now) enabled.
bool allow_peer(CurrentDevice& cur, int dev, int peer) {
    cur.use(dev);
    const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaSuccess) return true;
    (void)cudaGetLastError();
    if (e == cudaErrorPeerAccessAlreadyEnabled) return true;
    if (e == cudaErrorPeerAccessUnsupported || e == cudaErrorTooManyPeers) return false;
    check(e, "cudaDeviceEnablePeerAccess");
    return false;
}

void quietly(const char* what, cudaError_t e) {
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        std::cerr << "PeerLink cleanup: " << what << ": " << cudaGetErrorString(e) << '\n';
    }
}

}  // namespace

bool p2p_disabled_by_env() {
    const char* v = std::getenv("P100_DISABLE_P2P");
    return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
}

const char* path_name(Path p) { return p == Path::Peer ? "Peer" : "Staged"; }

Topology probe() {
    Topology t;
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        (void)cudaGetLastError();
        return t;
    }
    check(e, "cudaGetDeviceCount");
    t.device_count = n;
    if (n == 0) return t;
    CurrentDevice cur;
    t.peer.assign(n, std::vector<PeerInfo>(n));
    for (int s = 0; s < n; ++s) {
        cudaDeviceProp prop{};
        check(cudaGetDeviceProperties(&prop, s), "cudaGetDeviceProperties");
        char bus[32] = {};
        check(cudaDeviceGetPCIBusId(bus, sizeof bus, s), "cudaDeviceGetPCIBusId");
        t.name.emplace_back(prop.name);
        t.pci_bus_id.emplace_back(bus);
        for (int d = 0; d < n; ++d) {
            if (d == s) continue;
            PeerInfo& info = t.peer[s][d];
            int access = 0, atomics = 0;
            check(cudaDeviceCanAccessPeer(&access, s, d), "cudaDeviceCanAccessPeer");
            check(cudaDeviceGetP2PAttribute(&info.perf_rank, cudaDevP2PAttrPerformanceRank, s, d),
                  "cudaDeviceGetP2PAttribute(rank)");
            check(cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, s, d),
                  "cudaDeviceGetP2PAttribute(atomics)");
            info.can_access = access != 0;
            info.native_atomics = atomics != 0;
        }
    }
    return t;
}

std::string describe(const Topology& t) {
    std::ostringstream os;
    os << "Devices: " << t.device_count << '\n';
    for (int i = 0; i < t.device_count; ++i) os << "  " << i << ": " << t.name.at(i) << "  PCI " << t.pci_bus_id.at(i) << '\n';
    os << "Peer matrix (row=src, column=dst; access/rank/native-atomics):\n  src\\dst";
    for (int d = 0; d < t.device_count; ++d) os << '\t' << d;
    os << '\n';
    for (int s = 0; s < t.device_count; ++s) {
        os << "  " << s;
        for (int d = 0; d < t.device_count; ++d) {
            if (s == d) {
                os << "\t-";
                continue;
            }
            const PeerInfo& p = t.peer.at(s).at(d);
            os << '\t' << (p.can_access ? "yes" : "no") << '/' << p.perf_rank << '/' << (p.native_atomics ? "yes" : "no");
        }
        os << '\n';
    }
    return os.str();
}

struct PeerLink::Impl {
    struct Slot {
        void* host = nullptr;
        cudaEvent_t filled = nullptr;    // on src: D2H into this buffer done
        cudaEvent_t drained = nullptr;   // on dst: H2D out of this buffer done
        bool filled_used = false, drained_used = false;
    };
    int src = 0, dst = 0;
    std::size_t chunk = 0;
    Path path = Path::Staged;
    Slot slot[2];
    cudaStream_t dst_stream = nullptr;
    cudaEvent_t done = nullptr;          // last copy complete (src for Peer, dst for Staged)
    bool done_used = false;

    ~Impl() {
        // Wait for this link's own outstanding work, then release it.
        try {
            CurrentDevice cur;
            cur.use(src);
            for (auto& s : slot)
                if (s.filled_used) quietly("sync filled", cudaEventSynchronize(s.filled));
            cur.use(dst);
            for (auto& s : slot)
                if (s.drained_used) quietly("sync drained", cudaEventSynchronize(s.drained));
            cur.use(path == Path::Peer ? src : dst);
            if (done_used) quietly("sync done", cudaEventSynchronize(done));
            if (done) quietly("destroy done", cudaEventDestroy(done));
            cur.use(src);
            for (auto& s : slot)
                if (s.filled) quietly("destroy filled", cudaEventDestroy(s.filled));
            cur.use(dst);
            for (auto& s : slot)
                if (s.drained) quietly("destroy drained", cudaEventDestroy(s.drained));
            if (dst_stream) quietly("destroy stream", cudaStreamDestroy(dst_stream));
            for (auto& s : slot)
                if (s.host) quietly("free host", cudaFreeHost(s.host));
            // Peer access stays enabled: other code may rely on it.
        } catch (const std::exception& e) {
            std::cerr << "PeerLink cleanup: " << e.what() << '\n';
        }
    }
};

PeerLink::PeerLink(int src_dev, int dst_dev, std::size_t chunk_bytes) {
    if (chunk_bytes == 0) throw std::invalid_argument("PeerLink chunk_bytes must be nonzero");
    CurrentDevice cur;
    cur.use(src_dev);   // both ordinals are validated even for a staged link
    cur.use(dst_dev);
    impl_ = std::make_unique<Impl>();
    Impl& m = *impl_;
    m.src = src_dev;
    m.dst = dst_dev;
    m.chunk = chunk_bytes;
    if (src_dev != dst_dev && !p2p_disabled_by_env()) {
        int fwd = 0, rev = 0;
        check(cudaDeviceCanAccessPeer(&fwd, dst_dev, src_dev), "cudaDeviceCanAccessPeer");
        check(cudaDeviceCanAccessPeer(&rev, src_dev, dst_dev), "cudaDeviceCanAccessPeer");
        if (fwd && rev && allow_peer(cur, dst_dev, src_dev) && allow_peer(cur, src_dev, dst_dev)) m.path = Path::Peer;
    }
    if (m.path == Path::Staged) {
        cur.use(dst_dev);
        check(cudaStreamCreateWithFlags(&m.dst_stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        for (auto& s : m.slot) {
            check(cudaHostAlloc(&s.host, chunk_bytes, cudaHostAllocPortable), "cudaHostAlloc");
            check(cudaEventCreateWithFlags(&s.drained, cudaEventDisableTiming), "cudaEventCreate");
        }
        cur.use(src_dev);
        for (auto& s : m.slot) check(cudaEventCreateWithFlags(&s.filled, cudaEventDisableTiming), "cudaEventCreate");
        cur.use(dst_dev);
    } else {
        cur.use(src_dev);
    }
    check(cudaEventCreateWithFlags(&m.done, cudaEventDisableTiming), "cudaEventCreate");
    std::clog << "PeerLink " << src_dev << "->" << dst_dev << " path=" << path_name(m.path) << '\n';
}

PeerLink::~PeerLink() = default;

Path PeerLink::path() const { return impl_->path; }

void PeerLink::copy_async(void* dst, const void* src, std::size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return;
    Impl& m = *impl_;
    CurrentDevice cur;
    cur.use(m.src);
    if (m.path == Path::Peer) {
        // Chain behind this link's previous copy, whatever stream it used.
        if (m.done_used) check(cudaStreamWaitEvent(stream, m.done, 0), "cudaStreamWaitEvent");
        check(cudaMemcpyPeerAsync(dst, m.dst, src, m.src, bytes, stream), "cudaMemcpyPeerAsync");
        check(cudaEventRecord(m.done, stream), "cudaEventRecord");
        m.done_used = true;
        return;
    }
    const char* from = static_cast<const char*>(src);
    char* to = static_cast<char*>(dst);
    unsigned turn = 0;
    for (std::size_t off = 0; off < bytes;) {
        const std::size_t n = std::min(m.chunk, bytes - off);
        Impl::Slot& s = m.slot[turn++ % 2];
        // The buffer is reusable once its previous host->device copy drained.
        if (s.drained_used) check(cudaEventSynchronize(s.drained), "cudaEventSynchronize");
        cur.use(m.src);
        check(cudaMemcpyAsync(s.host, from + off, n, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(D2H)");
        check(cudaEventRecord(s.filled, stream), "cudaEventRecord");
        s.filled_used = true;
        cur.use(m.dst);
        check(cudaStreamWaitEvent(m.dst_stream, s.filled, 0), "cudaStreamWaitEvent");
        check(cudaMemcpyAsync(to + off, s.host, n, cudaMemcpyHostToDevice, m.dst_stream), "cudaMemcpyAsync(H2D)");
        check(cudaEventRecord(s.drained, m.dst_stream), "cudaEventRecord");
        s.drained_used = true;
        off += n;
    }
    check(cudaEventRecord(m.done, m.dst_stream), "cudaEventRecord");
    m.done_used = true;
    cur.use(m.src);
    check(cudaStreamWaitEvent(stream, m.done, 0), "cudaStreamWaitEvent");
}

}  // namespace p100::p2p

// ------------------------------------------------------------------ C view
struct p100_peer_link {
    p100::p2p::PeerLink link;
    p100_peer_link(int s, int d, std::size_t c) : link(s, d, c) {}
};

namespace {
template <class F>
p100_status guarded(F&& f) {
    p100b::clear_error();
    try {
        f();
        return P100_OK;
    } catch (const std::invalid_argument& e) {
        return p100b::set_error(P100_ERR_INVALID, "%s", e.what());
    } catch (const std::exception& e) {
        return p100b::set_error(P100_ERR_CUDA, "%s", e.what());
    }
}
}  // namespace

extern "C" {

size_t p100_p2p_describe(char* out, size_t out_len) {
    std::string text;
    if (guarded([&] { text = p100::p2p::describe(p100::p2p::probe()); })) return 0;
    if (out && out_len) std::snprintf(out, out_len, "%s", text.c_str());
    return text.size() + 1;
}

int p100_p2p_disabled_by_env(void) { return p100::p2p::p2p_disabled_by_env() ? 1 : 0; }

p100_status p100_peer_link_create(int src_dev, int dst_dev, size_t chunk_bytes, p100_peer_link** out) {
    if (!out) return p100b::set_error(P100_ERR_INVALID, "null out");
    *out = nullptr;
    return guarded([&] { *out = new p100_peer_link(src_dev, dst_dev, chunk_bytes); });
}

int p100_peer_link_path(const p100_peer_link* link) {
    return link->link.path() == p100::p2p::Path::Peer ? P100_PATH_PEER : P100_PATH_STAGED;
}

p100_status p100_peer_link_copy(p100_peer_link* link, void* dst, const void* src, size_t bytes, p100_stream_t stream) {
    if (!link) return p100b::set_error(P100_ERR_INVALID, "null link");
    return guarded([&] { link->link.copy_async(dst, src, bytes, stream); });
}

p100_status p100_peer_link_destroy(p100_peer_link* link) {
    return guarded([&] { delete link; });
}

}  // extern "C"
