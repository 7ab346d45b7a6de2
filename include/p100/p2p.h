// p100/p2p.h — peer-to-peer copy layer, C++ interface.
//
// Same interface as the reference's include/p100/p2p.h (Frostbite1536/P100),
// implemented by libp100_b200 (p100_b200/csrc/p2p.cpp) for one B200 box:
// every pair of GPUs reaches the other over NVLink/NVSwitch, so the Peer path
// is the normal one; the Staged path (pinned host double buffer) remains as
// the forced fallback (P100_DISABLE_P2P) and for same-device links.
// C callers use the p100_peer_link_* functions of p100/b200.h.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <memory>
#include <string>
#include <vector>

namespace p100::p2p {

struct PeerInfo {
    bool can_access = false;
    int perf_rank = -1;
    bool native_atomics = false;
};

struct Topology {
    int device_count = 0;
    std::vector<std::string> name, pci_bus_id;
    std::vector<std::vector<PeerInfo>> peer;   // [src][dst]
};

// Enumerates devices and peer capabilities; restores the current device.
Topology probe();
// Human-readable device list and peer matrix (access/rank/native-atomics).
std::string describe(const Topology& t);

enum class Path { Peer, Staged };
const char* path_name(Path p);
// True when P100_DISABLE_P2P is set to a non-empty value other than "0".
bool p2p_disabled_by_env();

class PeerLink {
public:
    PeerLink(int src_dev, int dst_dev, std::size_t chunk_bytes = 4u << 20);
    ~PeerLink();
    PeerLink(const PeerLink&) = delete;
    PeerLink& operator=(const PeerLink&) = delete;
    Path path() const;
    // stream belongs to src_dev.  Work already on the stream precedes the
    // copy; later work on the stream starts after the destination holds
    // every byte.  The host blocks only to reuse a pinned staging buffer.
    void copy_async(void* dst, const void* src, std::size_t bytes, cudaStream_t stream);

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace p100::p2p
