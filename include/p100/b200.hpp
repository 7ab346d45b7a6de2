// p100/b200.hpp — header-only C++ view of the B200 hot path (p100/b200.h).
//
// For C++ callers of the reference's numerics contract (include/p100/qmv.h,
// include/p100/attention.h): the same names and error behaviour, on device
// buffers.  Shape errors throw std::invalid_argument with the reference's
// wording (qmv_model.cpp:31,54; attention_reference.cpp:18-32); CUDA, NCCL,
// timeout and unsupported-device errors throw p100::cuda::Error, a
// std::runtime_error as P100_CUDA_CHECK throws (include/p100/check.h:7-17).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "p100/b200.h"

namespace p100::cuda {

class Error : public std::runtime_error {
public:
    Error(p100_status status, const std::string& what) : std::runtime_error(what), status_(status) {}
    p100_status status() const noexcept { return status_; }

private:
    p100_status status_;
};

inline void check(p100_status status) {
    if (status == P100_OK) return;
    const std::string text = p100_last_error();
    if (status == P100_ERR_INVALID) throw std::invalid_argument(text);
    throw Error(status, std::string(p100_status_name(status)) + ": " + text);
}

namespace qmv {

// Same order as p100::qmv::Type (include/p100/qmv.h:20).
enum class Type { q4_0 = P100_Q4_0, q8_0 = P100_Q8_0, q4_K = P100_Q4_K };

inline int block_size(Type t) { return p100_block_elems(static_cast<int>(t)); }
inline int block_bytes(Type t) { return p100_block_bytes(static_cast<int>(t)); }
inline std::size_t weight_bytes(Type t, int rows, int k) { return p100_weight_bytes(static_cast<int>(t), rows, k); }
inline std::size_t q8_1_bytes(int k, int batch = 1) { return p100_q8_1_bytes(k, batch); }

// Device counterpart of prepare()'s q8_1 fields for batch rows of k values.
inline void prepare(const float* x, void* x_q8_1, int k, int batch, cudaStream_t stream) {
    check(p100_q8_1_quantize(x, x_q8_1, k, batch, stream));
}

inline void dequantize(Type t, const void* w, int rows, int k, float* out, cudaStream_t stream) {
    check(p100_dequantize(static_cast<int>(t), w, rows, k, out, stream));
}

// Device counterpart of evaluate().q81 for a whole matrix: y[c*rows + r].
inline void mat_vec(Type t, const void* w, int rows, int k, const void* x_q8_1, int batch, float* y,
                    cudaStream_t stream, unsigned flags = 0) {
    check(p100_qmv_ex(static_cast<int>(t), w, rows, k, x_q8_1, batch, y, flags, stream));
}

}  // namespace qmv

// AttnParams-shaped descriptor with the decode split and KV-cache strides.
struct AttnDesc : p100_attn_desc {
    AttnDesc() : p100_attn_desc{1, 1, 1, 1, 1, 128, 128, 0.0f, 0.0f, 0, 0, 0, 0} {}
};

// validate(p, &why) of attention_reference.cpp:18-32.
inline bool validate(const p100_attn_desc& d, std::string* why = nullptr) {
    char buf[128] = {};
    const bool ok = p100_attn_validate(&d, buf, sizeof buf) == P100_OK;
    if (why) *why = buf;
    return ok;
}

// Owns a zero-initialised decode workspace sized for one descriptor.
class FaWorkspace {
public:
    FaWorkspace() = default;
    FaWorkspace(const p100_attn_desc& d, cudaStream_t stream) : bytes_(p100_fa_workspace_size(&d)) {
        if (bytes_ == 0) {
            const std::string why = p100_last_error();
            if (!why.empty()) throw std::invalid_argument(why);
            return;
        }
        if (cudaMalloc(&ptr_, bytes_) != cudaSuccess) {
            (void)cudaGetLastError();
            throw Error(P100_ERR_CUDA, "cudaMalloc(decode workspace) failed");
        }
        check(p100_fa_workspace_init(ptr_, bytes_, stream));
    }
    ~FaWorkspace() {
        if (ptr_) cudaFree(ptr_);
    }
    FaWorkspace(FaWorkspace&& o) noexcept : ptr_(std::exchange(o.ptr_, nullptr)), bytes_(o.bytes_) {}
    FaWorkspace& operator=(FaWorkspace&& o) noexcept {
        std::swap(ptr_, o.ptr_);
        std::swap(bytes_, o.bytes_);
        return *this;
    }
    FaWorkspace(const FaWorkspace&) = delete;
    FaWorkspace& operator=(const FaWorkspace&) = delete;
    void* data() const { return ptr_; }
    std::size_t size() const { return bytes_; }

private:
    void* ptr_ = nullptr;
    std::size_t bytes_ = 0;
};

// Split-K FA-vec decode (device counterpart of attention_reference for seq_q == 1).
inline void attention_decode(const p100_attn_desc& d, const float* q, const void* k, const void* v,
                             const float* mask, float* o, float* lse, const FaWorkspace& ws,
                             cudaStream_t stream) {
    check(p100_fa_decode(&d, q, k, v, mask, o, lse, ws.data(), ws.size(), stream));
}

// One rank of a row-split tensor-parallel group.
class TensorParallel {
public:
    static std::vector<unsigned char> unique_id() {
        std::vector<unsigned char> id(P100_TP_ID_BYTES);
        check(p100_tp_unique_id(id.data()));
        return id;
    }
    TensorParallel(const std::vector<unsigned char>& id, int nranks, int rank, int device) {
        check(p100_tp_init_rank(id.data(), nranks, rank, device, &tp_));
    }
    ~TensorParallel() {
        if (tp_) p100_tp_destroy(tp_);
    }
    TensorParallel(const TensorParallel&) = delete;
    TensorParallel& operator=(const TensorParallel&) = delete;
    int rank() const { return p100_tp_rank(tp_); }
    int size() const { return p100_tp_size(tp_); }
    void allreduce_sum(float* buf, std::size_t count, cudaStream_t stream) {
        check(p100_tp_allreduce_sum(tp_, buf, count, stream));
    }
    void allgather(const float* in, float* out, std::size_t count, cudaStream_t stream) {
        check(p100_tp_allgather(tp_, in, out, count, stream));
    }

private:
    p100_tp* tp_ = nullptr;
};

}  // namespace p100::cuda
