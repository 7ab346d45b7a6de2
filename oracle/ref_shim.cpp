// ref_shim.cpp — C entry points over the reference's own CPU contract.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified src/reference/*.cpp (from P100_REFERENCE_DIR)
// into oracle/_ref/libp100_ref.so.  The parity tests call it through ctypes
// to pin the restatement in p100_oracle.cpp against the reference itself;
// nothing in the product links it.
#include "p100/attention.h"
#include "p100/qmv.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <random>
#include <chrono>
#include <string>
#include <thread>
#include <vector>

namespace {
thread_local std::string g_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

p100::qmv::Type type_of(int t) {
    return t == 0 ? p100::qmv::Type::q4_0 : t == 1 ? p100::qmv::Type::q8_0 : p100::qmv::Type::q4_K;
}

// Field order shared with p100o_attn in p100_oracle.h.
struct attn_c {
    int batch, n_head_q, n_head_kv, seq_q, seq_kv, d_qk, d_v;
    float scale, softcap;
    int causal;
};
struct tiled_c {
    int br, bc;
    int qk_accum_fp16, p_fp16, o_fp16_out, qk_scale_in_q;
    float qk_q_prescale;
    int qk_products_fp16, qk_half2_chain;
    float kq_max_offset;
    int l_from_unrounded_p, o_accum_fp16, kv_parallel_blocks, o_accum_np;
    int o_accum_fp16_tile_flush;
};

p100::AttnParams params_of(const attn_c& a) {
    p100::AttnParams p;
    p.batch = a.batch; p.n_head_q = a.n_head_q; p.n_head_kv = a.n_head_kv;
    p.seq_q = a.seq_q; p.seq_kv = a.seq_kv; p.d_qk = a.d_qk; p.d_v = a.d_v;
    p.scale = a.scale; p.softcap = a.softcap; p.causal = a.causal != 0;
    return p;
}
}  // namespace

extern "C" {
const char* p100r_last_error(void) { return g_error.c_str(); }

float p100r_round_to_fp16(float x) { return p100::round_to_fp16(x); }
float p100r_round_to_fp16_d(double x) { return p100::round_to_fp16(x); }
uint16_t p100r_half_bits(float x) { return p100::qmv::half_bits(x); }
float p100r_half_value(uint16_t h) { return p100::qmv::half_value(h); }

void* p100r_rng_new(uint32_t seed) { return new std::mt19937(seed); }
void p100r_rng_free(void* r) { delete static_cast<std::mt19937*>(r); }

int p100r_random_row(int type, int k, void* rng, uint8_t* out) {
    return guarded([&] {
        const auto row = p100::qmv::random_row(type_of(type), k, *static_cast<std::mt19937*>(rng));
        std::memcpy(out, row.data(), row.size());
    });
}

// ActivationBlock is 68 four-byte fields; copied out verbatim.
int p100r_prepare(const float* x, int k, void* out) {
    static_assert(sizeof(p100::qmv::ActivationBlock) == 272, "ActivationBlock layout");
    return guarded([&] {
        const auto acts = p100::qmv::prepare(x, k);
        std::memcpy(out, acts.data(), acts.size() * sizeof(acts[0]));
    });
}

int p100r_evaluate(int type, const void* w, const float* x, int k, const void* acts_in, double* d3, float* f3) {
    return guarded([&] {
        const auto* a = static_cast<const p100::qmv::ActivationBlock*>(acts_in);
        const std::vector<p100::qmv::ActivationBlock> acts(a, a + k / 32);
        const auto r = p100::qmv::evaluate(type_of(type), w, x, k, acts);
        d3[0] = r.exact; d3[1] = r.h16_exact; d3[2] = r.weight_norm;
        f3[0] = r.q81; f3[1] = r.h8; f3[2] = r.h16;
    });
}

// prepare() of one activation row, then evaluate() of rows weight rows split
// over nthreads std::threads; q81 outputs to y.  Returns wall seconds
// (negative on error).  Used as the timed CPU baseline: it is the reference's
// own per-row CPU path, unmodified.
double p100r_evaluate_rows_threaded(int type, const void* w, int rows, int k, const float* x, float* y,
                                    int nthreads) {
    const auto start = std::chrono::steady_clock::now();
    std::vector<p100::qmv::ActivationBlock> acts;
    if (guarded([&] { acts = p100::qmv::prepare(x, k); })) return -1.0;
    const size_t row_bytes = size_t(k / p100::qmv::block_size(type_of(type))) *
                             p100::qmv::block_bytes(type_of(type));
    if (nthreads < 1) nthreads = 1;
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        pool.emplace_back([&, t] {
            for (int r = t; r < rows; r += nthreads)
                y[r] = p100::qmv::evaluate(type_of(type), static_cast<const uint8_t*>(w) + r * row_bytes, x, k,
                                           acts).q81;
        });
    }
    for (auto& th : pool) th.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
}

int p100r_validate(const void* a, char* why, int why_len) {
    std::string reason;
    const bool ok = p100::validate(params_of(*static_cast<const attn_c*>(a)), &reason);
    if (why && why_len > 0) {
        std::strncpy(why, reason.c_str(), size_t(why_len) - 1);
        why[why_len - 1] = 0;
    }
    return ok ? 1 : 0;
}

int p100r_attention_reference(const void* a, const float* q, const float* k, const float* v,
                              const float* mask, float* o, float* lse) {
    return guarded([&] {
        p100::attention_reference(params_of(*static_cast<const attn_c*>(a)), q, k, v, mask, o, lse);
    });
}

int p100r_attention_tiled(const void* a, const void* c, const float* q, const float* k, const float* v,
                          const float* mask, float* o, float* lse) {
    return guarded([&] {
        const auto& t = *static_cast<const tiled_c*>(c);
        p100::TiledModelConfig cfg;
        cfg.br = t.br; cfg.bc = t.bc;
        cfg.qk_accum_fp16 = t.qk_accum_fp16; cfg.p_fp16 = t.p_fp16; cfg.o_fp16_out = t.o_fp16_out;
        cfg.qk_scale_in_q = t.qk_scale_in_q; cfg.qk_q_prescale = t.qk_q_prescale;
        cfg.qk_products_fp16 = t.qk_products_fp16; cfg.qk_half2_chain = t.qk_half2_chain;
        cfg.kq_max_offset = t.kq_max_offset; cfg.l_from_unrounded_p = t.l_from_unrounded_p;
        cfg.o_accum_fp16 = t.o_accum_fp16; cfg.kv_parallel_blocks = t.kv_parallel_blocks;
        cfg.o_accum_np = t.o_accum_np; cfg.o_accum_fp16_tile_flush = t.o_accum_fp16_tile_flush;
        p100::attention_tiled_model(params_of(*static_cast<const attn_c*>(a)), cfg, q, k, v, mask, o, lse);
    });
}
}  // extern "C"
