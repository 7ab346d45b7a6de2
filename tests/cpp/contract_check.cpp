// contract_check.cpp — a C++ caller of include/p100/b200.hpp, the way a user
// of the reference's C++ contract would call the B200 path.
//
//   contract_check errors   no GPU needed: shape errors throw
//                           std::invalid_argument with the reference's text;
//                           valid calls without an sm_100 device throw
//                           p100::cuda::Error(P100_ERR_UNSUPPORTED).
//   contract_check gpu      Q8_1 prepare bit-exact, Q4_K mat-vec and a split
//                           FA decode against the oracle (oracle/lib).
// Exit 0 on success; prints PASS/FAIL lines like the reference's run_tests.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "p100/b200.hpp"
#include "../../oracle/p100_oracle.h"

namespace {
int failures = 0;
#define EXPECT(cond)                                                              \
    do {                                                                          \
        if (!(cond)) {                                                            \
            std::fprintf(stderr, "%s:%d: EXPECT(%s) failed\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                           \
        }                                                                         \
    } while (0)

template <class E, class F>
std::string throws(F&& f) {
    try {
        f();
    } catch (const E& e) {
        return e.what();
    }
    return "<no exception>";
}

void errors() {
    using p100::cuda::qmv::Type;
    EXPECT(throws<std::invalid_argument>([] { p100::cuda::qmv::prepare(nullptr, nullptr, 33, 1, nullptr); }) ==
           "whole activation blocks required");
    EXPECT(throws<std::invalid_argument>([] {
               p100::cuda::qmv::mat_vec(Type::q4_K, nullptr, 1, 128, nullptr, 1, nullptr, nullptr);
           }) == "whole weight blocks required");
    p100::cuda::AttnDesc d;
    d.n_head_q = 3;
    d.n_head_kv = 2;
    std::string why;
    EXPECT(!p100::cuda::validate(d, &why) && why == "n_head_q must be divisible by n_head_kv");
    d = p100::cuda::AttnDesc();
    d.softcap = -1;
    EXPECT(throws<std::invalid_argument>([&] { p100::cuda::FaWorkspace ws(d, nullptr); }) ==
           "softcap must be finite and non-negative");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        (void)cudaGetLastError();
        float x = 0;
        const std::string what = throws<p100::cuda::Error>([&] {
            p100::cuda::qmv::prepare(&x, &x, 32, 1, nullptr);
        });
        EXPECT(what.rfind("P100_ERR_UNSUPPORTED", 0) == 0);
    }
}

template <class T>
T* device_copy(const std::vector<T>& h) {
    T* d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

void gpu() {
    using p100::cuda::qmv::Type;
    cudaStream_t s;
    cudaStreamCreate(&s);
    std::mt19937 rng(600602);
    std::normal_distribution<float> normal(0, 1);
    const int k = 4096, rows = 17, batch = 2;
    std::vector<float> x(batch * k);
    for (auto& v : x) v = normal(rng);
    for (int i = 0; i < 32; ++i) x[i] = 0;
    // prepare: bit-exact
    float* dx = device_copy(x);
    std::vector<unsigned char> xq(p100::cuda::qmv::q8_1_bytes(k, batch)), want(xq.size());
    unsigned char* dxq = nullptr;
    cudaMalloc(&dxq, xq.size());
    p100::cuda::qmv::prepare(dx, dxq, k, batch, s);
    cudaMemcpyAsync(xq.data(), dxq, xq.size(), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    p100o_quantize_q8_1(x.data(), k, batch, want.data());
    EXPECT(xq == want);
    // Q4_K mat-vec within 1e-3 * ||w|| * ||x|| of the q81 model
    std::vector<unsigned char> w(p100::cuda::qmv::weight_bytes(Type::q4_K, rows, k));
    void* rg = p100o_rng_new(60060 + k + 2);
    const size_t rb = w.size() / rows;
    for (int r = 0; r < rows; ++r) p100o_random_row(P100O_Q4_K, k, rg, w.data() + r * rb);
    p100o_rng_free(rg);
    unsigned char* dw = device_copy(w);
    float* dy = nullptr;
    cudaMalloc(&dy, batch * rows * sizeof(float));
    p100::cuda::qmv::mat_vec(Type::q4_K, dw, rows, k, dxq, batch, dy, s);
    std::vector<float> y(batch * rows), yref(batch * rows), deq(size_t(rows) * k);
    cudaMemcpyAsync(y.data(), dy, y.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    std::vector<p100o_act> acts(batch * k / 32);
    for (int c = 0; c < batch; ++c) p100o_prepare(x.data() + c * k, k, acts.data() + c * k / 32);
    p100o_qmv_q81(P100O_Q4_K, w.data(), rows, k, acts.data(), batch, yref.data());
    p100o_dequantize(P100O_Q4_K, w.data(), rows, k, deq.data());
    for (int c = 0; c < batch; ++c) {
        double xn = 0;
        for (int i = 0; i < k; ++i) xn += double(x[c * k + i]) * x[c * k + i];
        for (int r = 0; r < rows; ++r) {
            double wn = 0;
            for (int i = 0; i < k; ++i) wn += double(deq[size_t(r) * k + i]) * deq[size_t(r) * k + i];
            EXPECT(std::fabs(double(y[c * rows + r]) - yref[c * rows + r]) <= 1e-3 * std::sqrt(wn * xn));
        }
    }
    // FA decode, 3 parts, against attention_reference
    p100::cuda::AttnDesc d;
    d.n_head_q = 8;
    d.n_head_kv = 2;
    d.seq_kv = 500;
    d.kv_splits = 3;
    std::vector<float> q(8 * 128), kv32(2 * 500 * 128 * 2);
    for (auto& v : q) v = normal(rng);
    for (auto& v : kv32) v = p100o_fp16_round(0.5f * normal(rng));
    std::vector<uint16_t> kv16(kv32.size());
    for (size_t i = 0; i < kv32.size(); ++i) kv16[i] = p100o_fp16_bits(kv32[i]);
    float* dq = device_copy(q);
    uint16_t* dkv = device_copy(kv16);
    float *dout = nullptr, *dlse = nullptr;
    cudaMalloc(&dout, 8 * 128 * sizeof(float));
    cudaMalloc(&dlse, 8 * sizeof(float));
    p100::cuda::FaWorkspace ws(d, s);
    p100::cuda::attention_decode(d, dq, dkv, dkv + 2 * 500 * 128, nullptr, dout, dlse, ws, s);
    std::vector<float> o(8 * 128), lse(8), oref(8 * 128), lref(8);
    cudaMemcpyAsync(o.data(), dout, o.size() * 4, cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(lse.data(), dlse, lse.size() * 4, cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    p100o_attn p{1, 8, 2, 1, 500, 128, 128, 0.0f, 0.0f, 0};
    p100o_attention_reference(&p, q.data(), kv32.data(), kv32.data() + 2 * 500 * 128, nullptr, oref.data(), lref.data());
    for (size_t i = 0; i < o.size(); ++i) EXPECT(std::fabs(o[i] - oref[i]) <= 1e-3 + 2e-3 * std::fabs(oref[i]));
    for (int i = 0; i < 8; ++i) EXPECT(std::fabs(lse[i] - lref[i]) <= 1e-3);
    for (void* ptr : {(void*)dx, (void*)dxq, (void*)dw, (void*)dy, (void*)dq, (void*)dkv, (void*)dout, (void*)dlse})
        cudaFree(ptr);
    cudaStreamDestroy(s);
}
}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "errors";
    try {
        if (mode == "errors") errors();
        else if (mode == "gpu") gpu();
        else {
            std::fprintf(stderr, "usage: contract_check errors|gpu\n");
            return 2;
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        ++failures;
    }
    std::printf("%s %s\n", failures ? "FAIL" : "PASS", mode.c_str());
    return failures ? 1 : 0;
}
