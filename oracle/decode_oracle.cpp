// decode_oracle.cpp — CPU restatement of the decode-step glue and of one
// batch-1 decode step.  TEST INFRASTRUCTURE ONLY: the parity tests call it as
// the checker of p100_b200/csrc/decode.cuh and decoder.cuh; nothing in the
// library calls it.
//
// The reference has no decode step (its contract is one mat-vec and one
// attention call: qmv_model.cpp, attention_reference.cpp), so parity here is
// against this restatement, written from the Llama-3 decode math, not pinned
// by reference golden vectors.  The glue functions repeat the GPU kernels'
// floating-point operations in the same order (compiled with
// -ffp-contract=off; std::fma where the kernel uses fmaf), so they are
// bit-exact targets.  The whole step reuses the pinned pieces (prepare's
// Q8_1, the q81 mat-vec of qmv_model.cpp:147-180, attention_reference of
// attention_reference.cpp:87-135 in FP64), so it is a tolerance target.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <initializer_list>
#include <utility>
#include <vector>

#include "p100_oracle.h"

namespace {

// Q8_1 of one 32-value block, as prepare() (qmv_model.cpp:53-71) forms it
// and packed {fp16 d, fp16 sum, int8 q[32]}.
void q8_1_block(const float* v, uint8_t* out) {
    p100o_act a;
    p100o_prepare(v, 32, &a);
    p100o_pack_q8_1(&a, 1, out);
}

// XOR butterfly 16, 8, 4, 2, 1 over 32 lanes: the value every lane holds.
float butterfly32(const float* in) {
    float v[32];
    std::memcpy(v, in, sizeof v);
    for (int off = 16; off > 0; off >>= 1) {
        float n[32];
        for (int l = 0; l < 32; ++l) n[l] = v[l] + v[l ^ off];
        std::memcpy(v, n, sizeof v);
    }
    return v[0];
}

uint16_t half_bits(float x) { return p100o_fp16_bits(x); }
float half_value(uint16_t h) { return p100o_fp16_value(h); }

std::vector<p100o_act> unpack_q8_1(const uint8_t* q, int k) {
    std::vector<p100o_act> acts(size_t(k / 32));
    for (int b = 0; b < k / 32; ++b) {
        const uint8_t* blk = q + size_t(b) * 36;
        p100o_act& a = acts[b];
        std::memset(&a, 0, sizeof a);
        a.qd = half_value(uint16_t(blk[0] | (blk[1] << 8)));
        a.qsum = half_value(uint16_t(blk[2] | (blk[3] << 8)));
        for (int i = 0; i < 32; ++i) a.q[i] = int8_t(blk[4 + i]);
    }
    return acts;
}

}  // namespace

extern "C" {

int p100o_rmsnorm_q8_1(float* x, const float* delta, const float* w, float eps, int k, void* out_q81, float* y_out) {
    if (k <= 0 || k % 32) return -1;
    // thread t of 1024 owns the float4 chunks c = t, t + 1024, ...
    constexpr int kThreads = 1024;
    if (delta)
        for (int i = 0; i < k; ++i) x[i] = x[i] + delta[i];
    std::vector<float> part(kThreads, 0.f);
    for (int t = 0; t < kThreads; ++t) {
        float s = 0.f;
        for (int c = t; c < k / 4; c += kThreads)
            for (int e = 0; e < 4; ++e) s = std::fma(x[4 * c + e], x[4 * c + e], s);
        part[t] = s;
    }
    float total = 0.f;
    for (int wp = 0; wp < kThreads / 32; ++wp) {
        const float ws = butterfly32(part.data() + wp * 32);
        total = wp == 0 ? ws : total + ws;
    }
    const float r = 1.0f / std::sqrt(total / float(k) + eps);
    uint8_t* out = static_cast<uint8_t*>(out_q81);
    std::vector<float> y(static_cast<size_t>(k));
    for (int i = 0; i < k; ++i) y[i] = (x[i] * r) * w[i];
    if (y_out) std::memcpy(y_out, y.data(), size_t(k) * 4);
    for (int b = 0; b < k / 32; ++b) q8_1_block(y.data() + size_t(b) * 32, out + size_t(b) * 36);
    return 0;
}

int p100o_rope_kv_append(float* qkv, int nq, int nkv, int hd, const float* rope_cs, int max_pos, int pos,
                         uint16_t* k_cache, uint16_t* v_cache, long long head_stride) {
    if (pos < 0 || pos >= max_pos || hd % 2) return -1;
    for (int h = 0; h < nq + 2 * nkv; ++h)
        for (int i = 0; i < hd / 2; ++i) {
            float* v = qkv + size_t(h) * hd + 2 * i;
            const float x0 = v[0], x1 = v[1];
            if (h >= nq + nkv) {
                uint16_t* dst = v_cache + (h - nq - nkv) * head_stride + size_t(pos) * hd + 2 * i;
                dst[0] = half_bits(x0);
                dst[1] = half_bits(x1);
                continue;
            }
            const float c = rope_cs[(size_t(pos) * (hd / 2) + i) * 2], s = rope_cs[(size_t(pos) * (hd / 2) + i) * 2 + 1];
            const float y0 = x0 * c - x1 * s;
            const float y1 = x0 * s + x1 * c;
            if (h < nq) {
                v[0] = y0;
                v[1] = y1;
            } else {
                uint16_t* dst = k_cache + (h - nq) * head_stride + size_t(pos) * hd + 2 * i;
                dst[0] = half_bits(y0);
                dst[1] = half_bits(y1);
            }
        }
    return 0;
}

// exp by Cody-Waite reduction and a degree-8 Taylor polynomial; the same
// steps as dec_exp in decode.cuh.
float p100o_dec_exp(float x) {
    if (x < -104.0f) return 0.0f;
    if (x > 89.0f) return INFINITY;
    const float n = std::rint(x * 1.44269504088896341f);
    const float r = std::fma(-n, 1.42860677e-06f, std::fma(-n, 0.693145751953125f, x));
    float p = 2.48015873e-05f;
    p = std::fma(p, r, 1.98412698e-04f);
    p = std::fma(p, r, 1.38888889e-03f);
    p = std::fma(p, r, 8.33333333e-03f);
    p = std::fma(p, r, 4.16666667e-02f);
    p = std::fma(p, r, 1.66666667e-01f);
    p = std::fma(p, r, 0.5f);
    p = std::fma(p, r, 1.0f);
    p = std::fma(p, r, 1.0f);
    const int ni = static_cast<int>(n);
    const int n1 = ni / 2, n2 = ni - n1;
    float s1, s2;
    const uint32_t b1 = uint32_t(n1 + 127) << 23, b2 = uint32_t(n2 + 127) << 23;
    std::memcpy(&s1, &b1, 4);
    std::memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

int p100o_swiglu_q8_1(const float* gu, int n, void* out_q81) {
    if (n <= 0 || n % 32) return -1;
    std::vector<float> h(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
        const float g = gu[i], u = gu[n + i];
        const float silu = g / (1.0f + p100o_dec_exp(-g));
        h[i] = silu * u;
    }
    uint8_t* out = static_cast<uint8_t*>(out_q81);
    for (int b = 0; b < n / 32; ++b) q8_1_block(h.data() + size_t(b) * 32, out + size_t(b) * 36);
    return 0;
}

int p100o_argmax(const float* x, int n, float* val) {
    float bv = -INFINITY;
    int bi = -1;
    for (int i = 0; i < n; ++i)
        if (x[i] > bv) {   // strict: the lowest index wins ties; NaN never wins
            bv = x[i];
            bi = i;
        }
    if (val) *val = bv;
    return bi < 0 ? 0 : bi;
}

int p100o_decode_step(const p100o_llama* c, const p100o_llama_weights* w, uint16_t* k_cache, uint16_t* v_cache,
                      const float* rope_cs, int pos, int token, float* logits, float* hidden_out) {
    return p100o_decode_step_kv(c, w, P100O_KV_F16, 1, k_cache, v_cache, rope_cs, pos, token, logits, hidden_out);
}

// With a q8_0 / q4_0 cache ([layer][n_head_kv][max_ctx][head_dim/32 blocks]):
// q and k rotated as p100o_rope_kv_append rotates them, the rotated k row and
// the v row of each kv head quantised into cache row pos (p100o_kv_quantize:
// ggml's block quantisers), attention over the rows converted to fp16
// (p100o_kv_to_f16), in FP64 as for an fp16 cache.  append = 0 (quantised
// caches only) leaves row pos as the caller gave it: a test then attends over
// the device's own new rows, whose codes can sit one rounding step away from
// these (the two sides' k and v differ in the last bits).
int p100o_decode_step_kv(const p100o_llama* c, const p100o_llama_weights* w, int kv_type, int append, void* k_cache,
                         void* v_cache, const float* rope_cs, int pos, int token, float* logits, float* hidden_out) {
    const int hd = c->head_dim, H = c->hidden;
    const int nq = c->n_head, nkv = c->n_head_kv, F = c->ffn;
    if (pos < 0 || pos >= c->max_ctx || token < 0 || token >= c->vocab) return -1;
    const long long hs = static_cast<long long>(c->max_ctx) * hd;
    // format of tensor id i: 0 embed, 1 lm_head, 2 + 7 * layer + {q k v o gate up down}
    auto tt = [&](int i) { return c->tensor_types ? c->tensor_types[i] : c->wtype; };
    auto lt = [&](int l, int part) { return tt(2 + 7 * l + part); };
    const int te = tt(0);
    const size_t rb_h = size_t(H / p100o_block_elems(te)) * p100o_block_bytes(te);
    std::vector<float> x(static_cast<size_t>(H)), delta(static_cast<size_t>(H));
    std::vector<uint8_t> xq(size_t(std::max(H, std::max(nq * hd, F)) / 32) * 36);
    std::vector<float> qkv(size_t(nq + 2 * nkv) * hd), attn(size_t(nq) * hd), gu(size_t(2) * F);
    if (p100o_dequantize(te, static_cast<const uint8_t*>(w->embed) + size_t(token) * rb_h, 1, H, x.data()))
        return -1;
    // y = m . xq (k inputs) over row ranges {format, rows} stored one after the other
    auto qmv = [&](const void* m, std::initializer_list<std::pair<int, int>> ranges, int k, float* y) {
        const std::vector<p100o_act> acts = unpack_q8_1(xq.data(), k);
        const uint8_t* p = static_cast<const uint8_t*>(m);
        for (const auto& r : ranges) {
            if (p100o_qmv_q81(r.first, p, r.second, k, acts.data(), 1, y)) return -1;
            p += size_t(r.second) * size_t(k / p100o_block_elems(r.first)) * p100o_block_bytes(r.first);
            y += r.second;
        }
        return 0;
    };
    for (int l = 0; l < c->n_layer; ++l) {
        p100o_rmsnorm_q8_1(x.data(), l == 0 ? nullptr : delta.data(), w->attn_norm[l], c->norm_eps, H, xq.data(),
                           nullptr);
        if (qmv(w->wqkv[l], {{lt(l, 0), nq * hd}, {lt(l, 1), nkv * hd}, {lt(l, 2), nkv * hd}}, H, qkv.data()))
            return -1;
        const size_t layer_off = size_t(l) * nkv * hs;
        const int seq = pos + 1;
        std::vector<float> kf(size_t(nkv) * seq * hd), vf(size_t(nkv) * seq * hd);
        if (kv_type == P100O_KV_F16) {
            uint16_t* kc = static_cast<uint16_t*>(k_cache);
            uint16_t* vc = static_cast<uint16_t*>(v_cache);
            p100o_rope_kv_append(qkv.data(), nq, nkv, hd, rope_cs, c->max_ctx, pos, kc + layer_off, vc + layer_off,
                                 hs);
            for (int h = 0; h < nkv; ++h)
                for (int j = 0; j < seq; ++j)
                    for (int e = 0; e < hd; ++e) {
                        const size_t src = layer_off + size_t(h) * hs + size_t(j) * hd + e;
                        kf[(size_t(h) * seq + j) * hd + e] = half_value(kc[src]);
                        vf[(size_t(h) * seq + j) * hd + e] = half_value(vc[src]);
                    }
        } else {
            const int bb = p100o_kv_block_bytes(kv_type);
            if (!bb || hd % 32) return -1;
            const size_t rb = size_t(hd / 32) * bb, hsb = size_t(c->max_ctx) * rb;
            uint8_t* kc = static_cast<uint8_t*>(k_cache) + size_t(l) * nkv * hsb;
            uint8_t* vc = static_cast<uint8_t*>(v_cache) + size_t(l) * nkv * hsb;
            std::vector<float> kr(static_cast<size_t>(hd));
            for (int h = 0; h < nq + nkv; ++h) {
                float* v = qkv.data() + size_t(h) * hd;
                for (int i = 0; i < hd / 2; ++i) {
                    const float x0 = v[2 * i], x1 = v[2 * i + 1];
                    const float cs = rope_cs[(size_t(pos) * (hd / 2) + i) * 2];
                    const float sn = rope_cs[(size_t(pos) * (hd / 2) + i) * 2 + 1];
                    float* out = h < nq ? v : kr.data();
                    out[2 * i] = x0 * cs - x1 * sn;
                    out[2 * i + 1] = x0 * sn + x1 * cs;
                }
                if (h >= nq && append) {
                    const int kh = h - nq;
                    p100o_kv_quantize(kv_type, kr.data(), size_t(hd), kc + kh * hsb + size_t(pos) * rb);
                    p100o_kv_quantize(kv_type, qkv.data() + size_t(nq + nkv + kh) * hd, size_t(hd),
                                      vc + kh * hsb + size_t(pos) * rb);
                }
            }
            std::vector<uint16_t> k16(size_t(seq) * hd), v16(size_t(seq) * hd);
            for (int h = 0; h < nkv; ++h) {
                p100o_kv_to_f16(kv_type, kc + h * hsb, hd, seq, 1, 1, hd / 32, 0, 0, k16.data());
                p100o_kv_to_f16(kv_type, vc + h * hsb, hd, seq, 1, 1, hd / 32, 0, 0, v16.data());
                for (size_t i = 0; i < k16.size(); ++i) {
                    kf[size_t(h) * seq * hd + i] = half_value(k16[i]);
                    vf[size_t(h) * seq * hd + i] = half_value(v16[i]);
                }
            }
        }
        // attention over rows [0, pos] of this layer's cache, in FP64
        p100o_attn ap = {1, nq, nkv, 1, seq, hd, hd, 0.0f, 0.0f, 0};
        if (p100o_attention_reference(&ap, qkv.data(), kf.data(), vf.data(), nullptr, attn.data(), nullptr))
            return -1;
        if (p100o_quantize_q8_1(attn.data(), nq * hd, 1, xq.data())) return -1;
        if (qmv(w->wo[l], {{lt(l, 3), H}}, nq * hd, delta.data())) return -1;
        p100o_rmsnorm_q8_1(x.data(), delta.data(), w->ffn_norm[l], c->norm_eps, H, xq.data(), nullptr);
        if (qmv(w->wgu[l], {{lt(l, 4), F}, {lt(l, 5), F}}, H, gu.data())) return -1;
        p100o_swiglu_q8_1(gu.data(), F, xq.data());
        if (qmv(w->wdown[l], {{lt(l, 6), H}}, F, delta.data())) return -1;
    }
    p100o_rmsnorm_q8_1(x.data(), delta.data(), w->out_norm, c->norm_eps, H, xq.data(), nullptr);
    if (hidden_out) std::memcpy(hidden_out, x.data(), size_t(H) * 4);
    if (qmv(w->lm_head, {{tt(1), c->vocab}}, H, logits)) return -1;
    return p100o_argmax(logits, c->vocab, nullptr);
}

}  // extern "C"
