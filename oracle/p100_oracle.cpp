// p100_oracle.cpp — CPU restatement of the P100 numerics contract.
//
// TEST INFRASTRUCTURE ONLY (see p100_oracle.h).  Compiled with
// -O2 -ffp-contract=off like the reference (src/reference/CMakeLists.txt:6):
// every expression below keeps the reference's operand order and precision,
// because the parity tests demand bit-identical results.
#include "p100_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <random>
#include <string>
#include <thread>
#include <chrono>
#include <vector>

namespace {

thread_local std::string g_error;

int fail(const char* why) {
    g_error = why;
    return -1;
}

// ---------------------------------------------------------------- binary16
// Round a finite double to the nearest binary16, ties to even, returning the
// half bit pattern.  Every float is exactly a double, so this one routine
// serves both overloads of round_to_fp16 (attention_reference.cpp:34-85 and
// attention_tiled_model.cpp:14-50) without a double rounding.
uint16_t half_from_double(double x) {
    uint64_t bits;
    std::memcpy(&bits, &x, sizeof bits);
    const uint16_t sign = static_cast<uint16_t>((bits >> 48) & 0x8000u);
    const int biased = static_cast<int>((bits >> 52) & 0x7ff);
    const uint64_t fraction = bits & ((1ull << 52) - 1);
    if (biased == 0x7ff) return sign | 0x7c00u | (fraction ? 0x200u : 0u);
    if (biased == 0) return sign;                 // |x| < 2^-1022 rounds to zero
    const int e = biased - 1023;                  // x = 1.f * 2^e
    if (e > 15) return sign | 0x7c00u;            // beyond 65504 + half an ulp
    const uint64_t significand = fraction | (1ull << 52);
    // Normal halves keep 11 significant bits; subnormals count units of 2^-24.
    const int shift = e >= -14 ? 42 : 28 - e;
    if (shift > 63) return sign;
    uint64_t kept = significand >> shift;
    const uint64_t rest = significand & ((1ull << shift) - 1);
    const uint64_t midpoint = 1ull << (shift - 1);
    if (rest > midpoint || (rest == midpoint && (kept & 1u))) ++kept;
    if (e >= -14) {
        // A carry out of the significand steps the exponent (65520 -> inf).
        return sign | static_cast<uint16_t>((static_cast<uint32_t>(e + 15) << 10) + kept - 1024u);
    }
    return sign | static_cast<uint16_t>(kept);    // 1024 here is the smallest normal
}

float half_to_float(uint16_t h) {
    const int e = (h >> 10) & 31;
    const int m = h & 1023;
    float magnitude;
    if (e == 31) magnitude = m ? std::numeric_limits<float>::quiet_NaN() : std::numeric_limits<float>::infinity();
    else if (e == 0) magnitude = std::ldexp(static_cast<float>(m), -24);
    else magnitude = std::ldexp(static_cast<float>(m | 1024), e - 25);
    return (h & 0x8000u) ? -magnitude : magnitude;
}

// round_to_fp16(float): non-finite values pass through unchanged
// (attention_reference.cpp:42).
float fp16_round(float x) {
    if (!std::isfinite(x)) return x;
    return half_to_float(half_from_double(x));
}

// round_to_fp16(double) (attention_tiled_model.cpp:14-50).
float fp16_round_d(double x) {
    if (!std::isfinite(x)) return static_cast<float>(x);
    return half_to_float(half_from_double(x));
}

// ---------------------------------------------------------------- formats
// Q5_K (176 bytes) and Q6_K (210 bytes) are ggml's published super-block
// formats; the reference's contract has the first three only.
int elems_of(int t) { return t == P100O_Q4_0 || t == P100O_Q8_0 ? 32 : 256; }   // qmv_model.cpp:12
int bytes_of(int t) {                                                           // :13
    return t == P100O_Q4_0 ? 18 : t == P100O_Q8_0 ? 34 : t == P100O_Q4_K ? 144 : t == P100O_Q5_K ? 176 : 210;
}
bool ref_type(int t) { return t == P100O_Q4_0 || t == P100O_Q8_0 || t == P100O_Q4_K; }
bool known_type(int t) { return ref_type(t) || t == P100O_Q5_K || t == P100O_Q6_K; }

// 0,2,1,3 order inside each group of four (qmv_model.cpp:64).
inline int lane_order(int i) { return (i & ~3) | ((i & 1) << 1) | ((i & 2) >> 1); }

// XOR butterfly over 32 lanes with offsets 16..1, FP32 rounding at each level
// (qmv_model.cpp:45-52).
float butterfly_sum(const float* in) {
    float a[32], b[32];
    std::copy(in, in + 32, a);
    for (int off = 16; off > 0; off >>= 1) {
        for (int i = 0; i < 32; ++i) b[i] = a[i] + a[i ^ off];
        std::copy(b, b + 32, a);
    }
    return a[0];
}

// One 32-value slab of a weight block: the record of qmv_model.cpp:78-91
// (value d*sc*q - m*mn); Q6_K scales each 16 values, so sc2 is the scale of
// values 16..31 (equal to sc for every other type).
struct Slab {
    float d = 0, m = 0;
    int sc = 1, mn = 0, sc2 = 1;
    int q[32];
};

// Six-bit scale/min unpacking of Q4_K (qmv_model.cpp:72-77).
void q4k_scale_min(const uint8_t* scales, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = scales[j] & 63;
        mn = scales[j + 4] & 63;
    } else {
        sc = (scales[j + 4] & 15) | ((scales[j - 4] >> 6) << 4);
        mn = (scales[j + 4] >> 4) | ((scales[j] >> 6) << 4);
    }
}

Slab slab_of(int t, const uint8_t* block, int sub) {
    Slab s;
    uint16_t d;
    std::memcpy(&d, block, 2);
    s.d = half_to_float(d);
    if (t == P100O_Q4_0) {
        // byte i%16, low nibble for i<16 and high nibble for i>=16, minus 8
        for (int i = 0; i < 32; ++i) s.q[i] = ((block[2 + (i & 15)] >> ((i >> 4) * 4)) & 15) - 8;
    } else if (t == P100O_Q8_0) {
        for (int i = 0; i < 32; ++i) s.q[i] = static_cast<int8_t>(block[2 + i]);
    } else if (t == P100O_Q4_K) {
        uint16_t dmin;
        std::memcpy(&dmin, block + 2, 2);
        s.m = half_to_float(dmin);
        q4k_scale_min(block + 4, sub, s.sc, s.mn);
        const uint8_t* qs = block + 16 + (sub / 2) * 32;
        for (int i = 0; i < 32; ++i) s.q[i] = (qs[i] >> ((sub % 2) * 4)) & 15;
    } else if (t == P100O_Q5_K) {
        // {d, dmin, scales[12], qh[32], qs[128]} (ggml block_q5_K): the Q4_K
        // nibble of slab `sub` plus 16 * bit `sub` of qh[i]
        uint16_t dmin;
        std::memcpy(&dmin, block + 2, 2);
        s.m = half_to_float(dmin);
        q4k_scale_min(block + 4, sub, s.sc, s.mn);
        const uint8_t* qh = block + 16;
        const uint8_t* qs = block + 48 + (sub / 2) * 32;
        for (int i = 0; i < 32; ++i) s.q[i] = ((qs[i] >> ((sub % 2) * 4)) & 15) | (((qh[i] >> sub) & 1) << 4);
    } else {
        // {ql[128], qh[64], int8 scales[16], d} (ggml block_q6_K): slab sub =
        // 4h + c of half h; low 4 bits from ql[64h + 32(c&1) + i] (high
        // nibble when c >= 2), bits 4-5 from qh[32h + i] >> 2c, minus 32;
        // scale scales[8h + 2c + i/16]
        uint16_t d;
        std::memcpy(&d, block + 208, 2);
        s.d = half_to_float(d);
        const int h = sub / 4, c = sub % 4;
        const uint8_t* ql = block + 64 * h + 32 * (c & 1);
        const uint8_t* qh = block + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(block + 192 + 8 * h + 2 * c);
        s.sc = sc[0];
        s.sc2 = sc[1];
        for (int i = 0; i < 32; ++i) s.q[i] = (((ql[i] >> ((c >> 1) * 4)) & 15) | (((qh[i] >> (2 * c)) & 3) << 4)) - 32;
        return s;
    }
    s.sc2 = s.sc;
    return s;
}

// Dequantised value in double, qmv_model.cpp:143.
inline double slab_value(const Slab& s, int i) {
    return double(s.d) * (i < 16 ? s.sc : s.sc2) * s.q[i] - double(s.m) * s.mn;
}

// h16 FP64 dot, qmv_model.cpp:92-99.
double h16_exact_slab(const Slab& w, const p100o_act& a) {
    double dot = 0;
    for (int i = 0; i < 32; ++i) dot += double(w.q[i]) * a.h[lane_order(i)];
    return double(w.d) * w.sc * a.scale * dot - double(w.m) * w.mn * a.scale * a.sum;
}

// Two interleaved half FMA chains, one FP16 rounding per FMA (qmv_model.cpp:109-119).
float h16_chain(const Slab& w, const p100o_act& a, int start, int chain) {
    float even = 0, odd = 0;
    for (int j = start; j < start + chain; ++j) {
        const int i = 2 * j;
        even = fp16_round_d(double(w.q[lane_order(i)]) * a.h[i] + even);
        odd = fp16_round_d(double(w.q[lane_order(i + 1)]) * a.h[i + 1] + odd);
    }
    return even + odd;
}

// qmv::h16_model (qmv_model.cpp:120-133).
float h16_model(int t, const uint8_t* w, int k, const p100o_act* acts, int chain) {
    float out = 0;
    const int bs = elems_of(t), bb = bytes_of(t);
    for (int b = 0; b < k / bs; ++b) {
        for (int sub = 0; sub < bs / 32; ++sub) {
            const Slab s = slab_of(t, w + b * bb, sub);
            const p100o_act& x = acts[b * bs / 32 + sub];
            const float ds = (s.d * s.sc) * x.scale;
            const float ms = (s.m * s.mn) * x.scale;
            for (int start = 0; start < 16; start += chain) out += h16_chain(s, x, start, chain) * ds;
            if (t == P100O_Q4_K) out -= ms * x.sum;
        }
    }
    return out;
}

// The q81 dot of one weight row against one prepared activation row
// (qmv_model.cpp:147-180), in the model's sequential FP32 order.
float q81_row(int t, const uint8_t* w, int k, const p100o_act* acts) {
    float r = 0;
    const int bs = elems_of(t), bb = bytes_of(t);
    if (!ref_type(t)) {
        // Q5_K / Q6_K, per 32-value slab against its Q8_1 block, in the
        // library's slab arithmetic (qmv.cuh slab_dot): Q5_K as Q4_K,
        // fma(d, qd * (dot * sc), -dmin * (qd * (sum(q8) * mn))); Q6_K
        // (d * qd) * (sc * dot(values 0..15) + sc2 * dot(values 16..31))
        for (int b = 0; b < k / bs; ++b)
            for (int sub = 0; sub < 8; ++sub) {
                const Slab s = slab_of(t, w + size_t(b) * bb, sub);
                const p100o_act& a = acts[b * 8 + sub];
                if (t == P100O_Q5_K) {
                    int dot = 0, sum = 0;
                    for (int i = 0; i < 32; ++i) {
                        dot += s.q[i] * a.q[i];
                        sum += a.q[i];
                    }
                    r += std::fma(s.d, a.qd * float(dot * s.sc), -s.m * (a.qd * float(sum * s.mn)));
                } else {
                    int lo = 0, hi = 0;
                    for (int i = 0; i < 16; ++i) {
                        lo += s.q[i] * a.q[i];
                        hi += s.q[i + 16] * a.q[i + 16];
                    }
                    r += (s.d * a.qd) * float(s.sc * lo + s.sc2 * hi);
                }
            }
        return r;
    }
    for (int b = 0; b < k / bs; ++b) {
        const uint8_t* block = w + b * bb;
        if (t != P100O_Q4_K) {
            const Slab s = slab_of(t, block, 0);
            const p100o_act& act = acts[b];
            const int calls = t == P100O_Q4_0 ? 2 : 4;
            for (int call = 0; call < calls; ++call) {
                int dot = 0;
                for (int i = 0; i < 8; ++i) {
                    const int j = call * 8 + i;
                    if (t == P100O_Q4_0) {
                        // unbiased nibbles; the -8 comes back through qsum
                        dot += (s.q[j] + 8) * act.q[j];
                        dot += (s.q[j + 16] + 8) * act.q[j + 16];
                    } else {
                        dot += s.q[j] * act.q[j];
                    }
                }
                if (t == P100O_Q4_0) r = std::fma(s.d, std::fma(float(dot), act.qd, -4.f * act.qsum), r);
                else r = std::fma(s.d * act.qd, float(dot), r);
            }
        } else {
            Slab s[8];
            for (int sub = 0; sub < 8; ++sub) s[sub] = slab_of(t, block, sub);
            for (int group = 0; group < 4; ++group) {
                for (int call = 0; call < 4; ++call) {
                    float sd = 0, sm = 0;
                    for (int z = 0; z < 2; ++z) {
                        const int sub = group * 2 + z;
                        const p100o_act& act = acts[b * 8 + sub];
                        int dot = 0, sum = 0;
                        for (int i = 0; i < 8; ++i) {
                            // elements call*4 .. +3 and call*4+16 .. +19
                            const int j = call * 4 + (i & 3) + (i >> 2) * 16;
                            dot += s[sub].q[j] * act.q[j];
                            sum += act.q[j];
                        }
                        sd = std::fma(act.qd, float(dot * s[sub].sc), sd);
                        sm = std::fma(act.qd, float(sum * s[sub].mn), sm);
                    }
                    r += std::fma(s[0].d, sd, -s[0].m * sm);
                }
            }
        }
    }
    return r;
}

bool check_qmv_shape(int t, int k) {
    if (!known_type(t)) {
        fail("unknown weight type");
        return false;
    }
    if (k <= 0 || k % elems_of(t)) {
        fail("whole weight blocks required");  // qmv_model.cpp:31
        return false;
    }
    return true;
}

// ---------------------------------------------------------------- attention
bool attn_valid(const p100o_attn& p, const char** reason) {
    // attention_reference.cpp:18-32, same reasons in the same order.
    *reason = nullptr;
    if (p.batch <= 0 || p.n_head_q <= 0 || p.n_head_kv <= 0 || p.seq_q <= 0 || p.seq_kv <= 0 ||
        p.d_qk <= 0 || p.d_v <= 0) {
        *reason = "all dimensions must be positive";
    } else if (p.n_head_q % p.n_head_kv != 0) {
        *reason = "n_head_q must be divisible by n_head_kv";
    } else if (p.softcap < 0.0f || !std::isfinite(p.softcap)) {
        *reason = "softcap must be finite and non-negative";
    } else if (!std::isfinite(p.scale)) {
        *reason = "scale must be finite";
    }
    return *reason == nullptr;
}

float effective_scale(const p100o_attn& p) {
    // attention_reference.cpp:14-16
    return p.scale == 0.0f ? 1.0f / std::sqrt(static_cast<float>(p.d_qk)) : p.scale;
}

// One (batch, query head) slice of attention_reference
// (attention_reference.cpp:95-133): FP64 logits, softmax and accumulation.
void reference_head(const p100o_attn& p, int b, int h, const float* q, const float* k,
                    const float* v, const float* mask, float* o, float* lse,
                    std::vector<double>& logits, std::vector<double>& acc) {
    const double scale = effective_scale(p);
    const double neg_inf = -std::numeric_limits<double>::infinity();
    const int kh = h / (p.n_head_q / p.n_head_kv);
    const size_t kv_base = (size_t(b) * p.n_head_kv + kh) * p.seq_kv;
    for (int i = 0; i < p.seq_q; ++i) {
        const size_t row = (size_t(b) * p.n_head_q + h) * p.seq_q + i;
        double m = neg_inf;
        for (int j = 0; j < p.seq_kv; ++j) {
            double x = neg_inf;
            const bool visible = !p.causal || j <= i + (p.seq_kv - p.seq_q);
            if (visible) {
                double dot = 0.0;
                for (int d = 0; d < p.d_qk; ++d)
                    dot += double(q[row * p.d_qk + d]) * k[(kv_base + j) * p.d_qk + d];
                x = dot * scale;
                if (p.softcap > 0.0f) x = p.softcap * std::tanh(x / p.softcap);
                if (mask) x += mask[size_t(i) * p.seq_kv + j];
            }
            logits[j] = x;
            m = std::max(m, x);
        }
        double sum = 0.0;
        std::fill(acc.begin(), acc.end(), 0.0);
        if (m != neg_inf) {
            for (int j = 0; j < p.seq_kv; ++j) {
                const double weight = std::exp(logits[j] - m);
                sum += weight;
                for (int d = 0; d < p.d_v; ++d) acc[d] += weight * v[(kv_base + j) * p.d_v + d];
            }
        }
        for (int d = 0; d < p.d_v; ++d)
            o[row * p.d_v + d] = sum == 0.0 ? 0.0f : static_cast<float>(acc[d] / sum);
        if (lse) lse[row] = sum == 0.0 ? static_cast<float>(neg_inf) : static_cast<float>(m + std::log(sum));
    }
}

}  // namespace

extern "C" {

const char* p100o_last_error(void) { return g_error.c_str(); }

float p100o_fp16_round(float x) { return fp16_round(x); }
float p100o_fp16_round_d(double x) { return fp16_round_d(x); }
// qmv::half_bits is the bit pattern of round_to_fp16(x) (qmv_model.cpp:14-22);
// NaN maps to a quiet NaN with the sign kept.
uint16_t p100o_fp16_bits(float x) { return half_from_double(x); }
float p100o_fp16_value(uint16_t h) { return half_to_float(h); }

int p100o_block_elems(int type) { return known_type(type) ? elems_of(type) : -1; }
int p100o_block_bytes(int type) { return known_type(type) ? bytes_of(type) : -1; }

int p100o_prepare(const float* x, int k, p100o_act* out) {
    // qmv::prepare, qmv_model.cpp:53-71
    if (k <= 0 || k % 32) return fail("whole activation blocks required");
    for (int b = 0; b < k / 32; ++b) {
        p100o_act& a = out[b];
        const float* xb = x + b * 32;
        a.scale = 0;
        for (int i = 0; i < 32; ++i) a.scale = std::max(a.scale, std::fabs(xb[i]));
        const float d = a.scale / 127.0f;
        float originals[32], rounded[32];
        for (int i = 0; i < 32; ++i) {
            originals[i] = xb[i];
            rounded[i] = fp16_round(a.scale == 0 ? 0.f : xb[i] / a.scale);
            a.h[lane_order(i)] = rounded[i];
            a.q[i] = a.scale == 0 ? 0 : int(std::round(xb[i] / d));
        }
        a.sum = butterfly_sum(rounded);
        a.qsum = fp16_round(butterfly_sum(originals));
        a.qd = fp16_round(d);
    }
    return 0;
}

void p100o_pack_q8_1(const p100o_act* a, int nblocks, void* out) {
    uint8_t* o = static_cast<uint8_t*>(out);
    for (int b = 0; b < nblocks; ++b) {
        const uint16_t d = half_from_double(a[b].qd), s = half_from_double(a[b].qsum);
        std::memcpy(o + 36 * b, &d, 2);
        std::memcpy(o + 36 * b + 2, &s, 2);
        for (int i = 0; i < 32; ++i) o[36 * b + 4 + i] = static_cast<uint8_t>(static_cast<int8_t>(a[b].q[i]));
    }
}

int p100o_quantize_q8_1(const float* x, int k, int batch, void* out) {
    if (batch <= 0) return fail("batch must be positive");
    std::vector<p100o_act> acts(k > 0 ? k / 32 : 0);
    for (int c = 0; c < batch; ++c) {
        if (p100o_prepare(x + size_t(c) * k, k, acts.data())) return -1;
        p100o_pack_q8_1(acts.data(), k / 32, static_cast<uint8_t*>(out) + size_t(c) * (k / 32) * 36);
    }
    return 0;
}

void* p100o_rng_new(uint32_t seed) { return new std::mt19937(seed); }
void p100o_rng_free(void* rng) { delete static_cast<std::mt19937*>(rng); }

int p100o_random_row(int type, int k, void* rng, uint8_t* out) {
    // qmv::random_row, qmv_model.cpp:30-43: every byte uniform, then finite
    // fp16 scales uniform in [0.002, 0.08) over the scale fields.
    if (!check_qmv_shape(type, k)) return -1;
    std::mt19937& g = *static_cast<std::mt19937*>(rng);
    std::uniform_real_distribution<float> scale(0.002f, 0.08f);
    std::uniform_int_distribution<int> byte(0, 255);
    const int bb = bytes_of(type);
    for (int b = 0; b < k / elems_of(type); ++b) {
        uint8_t* p = out + size_t(b) * bb;
        for (int i = 0; i < bb; ++i) p[i] = static_cast<uint8_t>(byte(g));
        const uint16_t d = half_from_double(scale(g));
        std::memcpy(p + (type == P100O_Q6_K ? 208 : 0), &d, 2);
        if (type == P100O_Q4_K || type == P100O_Q5_K) {
            const uint16_t m = half_from_double(scale(g));
            std::memcpy(p + 2, &m, 2);
        }
    }
    return 0;
}

void p100o_fill_normal(uint32_t seed, float mean, float stddev, int round_fp16, size_t n, float* out) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (size_t i = 0; i < n; ++i) {
        const float v = dist(rng);
        out[i] = round_fp16 ? fp16_round(v) : v;
    }
}

void p100o_fill_uniform(uint32_t seed, float lo, float hi, int round_fp16, size_t n, float* out) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (size_t i = 0; i < n; ++i) {
        const float v = dist(rng);
        out[i] = round_fp16 ? fp16_round(v) : v;
    }
}

int p100o_dequantize(int type, const void* w, int rows, int k, float* out) {
    if (!check_qmv_shape(type, k)) return -1;
    if (rows < 0) return fail("rows must be non-negative");
    const uint8_t* base = static_cast<const uint8_t*>(w);
    const int bs = elems_of(type), bb = bytes_of(type);
    const size_t row_bytes = size_t(k / bs) * bb;
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < k / bs; ++b) {
            for (int sub = 0; sub < bs / 32; ++sub) {
                const Slab s = slab_of(type, base + r * row_bytes + size_t(b) * bb, sub);
                for (int i = 0; i < 32; ++i)
                    out[size_t(r) * k + b * bs + sub * 32 + i] = static_cast<float>(slab_value(s, i));
            }
        }
    }
    return 0;
}

int p100o_evaluate(int type, const void* w_row, const float* x, int k, const p100o_act* acts,
                   p100o_eval* out) {
    // qmv::evaluate, qmv_model.cpp:134-185
    if (!check_qmv_shape(type, k)) return -1;
    const uint8_t* w = static_cast<const uint8_t*>(w_row);
    const int bs = elems_of(type), bb = bytes_of(type);
    p100o_eval r{};
    for (int b = 0; b < k / bs; ++b) {
        for (int sub = 0; sub < bs / 32; ++sub) {
            const Slab s = slab_of(type, w + b * bb, sub);
            const int base = b * bs + sub * 32;
            r.h16_exact += h16_exact_slab(s, acts[base / 32]);
            for (int i = 0; i < 32; ++i) {
                const double v = slab_value(s, i);
                r.exact += v * x[base + i];
                r.weight_norm += v * v;
            }
        }
    }
    r.q81 = q81_row(type, w, k, acts);
    r.weight_norm = std::sqrt(r.weight_norm);
    // the h16 model (one scale per 32 values) covers the reference's types
    r.h8 = ref_type(type) ? h16_model(type, w, k, acts, 8) : NAN;
    r.h16 = ref_type(type) ? h16_model(type, w, k, acts, 16) : NAN;
    if (!ref_type(type)) r.h16_exact = NAN;
    *out = r;
    return 0;
}

// qmv::h16_model (qmv_model.cpp:120-133) for every row and column,
// y[c*rows + r]; acts holds batch rows of k/32 blocks.
int p100o_qmv_h16(int type, const void* w, int rows, int k, const p100o_act* acts, int batch, int chain, float* y) {
    if (!check_qmv_shape(type, k)) return -1;
    if (rows < 0 || batch <= 0) return fail("rows must be non-negative and batch positive");
    if (chain != 8 && chain != 16) return fail("invalid h16 shape/chain");   // qmv_model.cpp:122
    if (!ref_type(type)) return fail("the h16 path covers Q4_0, Q8_0 and Q4_K");
    const size_t rb = size_t(k / elems_of(type)) * bytes_of(type);
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    for (int c = 0; c < batch; ++c)
        for (int r = 0; r < rows; ++r)
            y[size_t(c) * rows + r] = h16_model(type, wb + r * rb, k, acts + size_t(c) * (k / 32), chain);
    return 0;
}

int p100o_qmv_q81(int type, const void* w, int rows, int k, const p100o_act* acts, int batch, float* y) {
    if (!check_qmv_shape(type, k)) return -1;
    if (rows < 0 || batch <= 0) return fail("rows must be non-negative and batch positive");
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    const uint8_t* base = static_cast<const uint8_t*>(w);
    for (int c = 0; c < batch; ++c)
        for (int r = 0; r < rows; ++r)
            y[size_t(c) * rows + r] = q81_row(type, base + r * row_bytes, k, acts + size_t(c) * (k / 32));
    return 0;
}

double p100o_qmv_q81_threaded(int type, const void* w, int rows, int k, const p100o_act* acts,
                              int batch, float* y, int nthreads) {
    if (!check_qmv_shape(type, k) || rows < 0 || batch <= 0) return -1.0;
    if (nthreads < 1) nthreads = 1;
    const size_t row_bytes = size_t(k / elems_of(type)) * bytes_of(type);
    const uint8_t* base = static_cast<const uint8_t*>(w);
    const auto start = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        pool.emplace_back([=] {
            const int r0 = int(int64_t(rows) * t / nthreads), r1 = int(int64_t(rows) * (t + 1) / nthreads);
            for (int c = 0; c < batch; ++c)
                for (int r = r0; r < r1; ++r)
                    y[size_t(c) * rows + r] = q81_row(type, base + r * row_bytes, k, acts + size_t(c) * (k / 32));
        });
    }
    for (auto& th : pool) th.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
}

float p100o_attn_effective_scale(const p100o_attn* p) { return effective_scale(*p); }

int p100o_attn_validate(const p100o_attn* p, char* why, int why_len) {
    const char* reason;
    const bool ok = attn_valid(*p, &reason);
    if (why && why_len > 0) {
        std::snprintf(why, size_t(why_len), "%s", ok ? "" : reason);
    }
    return ok ? 1 : 0;
}

int p100o_attention_reference(const p100o_attn* p, const float* q, const float* k, const float* v,
                              const float* mask, float* o, float* lse) {
    const char* reason;
    if (!attn_valid(*p, &reason)) return fail(reason);
    std::vector<double> logits(p->seq_kv), acc(p->d_v);
    for (int b = 0; b < p->batch; ++b)
        for (int h = 0; h < p->n_head_q; ++h) reference_head(*p, b, h, q, k, v, mask, o, lse, logits, acc);
    return 0;
}

double p100o_attention_reference_threaded(const p100o_attn* p, const float* q, const float* k,
                                          const float* v, float* o, float* lse, int nthreads) {
    const char* reason;
    if (!attn_valid(*p, &reason)) {
        fail(reason);
        return -1.0;
    }
    if (nthreads < 1) nthreads = 1;
    const int heads = p->batch * p->n_head_q;
    const auto start = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        pool.emplace_back([=] {
            std::vector<double> logits(p->seq_kv), acc(p->d_v);
            for (int bh = t; bh < heads; bh += nthreads)
                reference_head(*p, bh / p->n_head_q, bh % p->n_head_q, q, k, v, nullptr, o, lse, logits, acc);
        });
    }
    for (auto& th : pool) th.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
}

int p100o_attention_tiled(const p100o_attn* pp, const p100o_tiled* cc, const float* q, const float* k,
                          const float* v, const float* mask, float* o, float* lse) {
    // attention_tiled_model, attention_tiled_model.cpp:52-227
    const p100o_attn& p = *pp;
    const p100o_tiled& cfg = *cc;
    const char* reason;
    if (!attn_valid(p, &reason)) return fail(reason);
    if (cfg.br <= 0 || cfg.bc <= 0) return fail("br and bc must be positive");
    if (cfg.kv_parallel_blocks < 1 || cfg.o_accum_np < 1)
        return fail("KV parallel blocks and O accumulator count must be positive");
    const int modes = (cfg.qk_accum_fp16 ? 1 : 0) + (cfg.qk_products_fp16 ? 1 : 0) + (cfg.qk_half2_chain > 0 ? 1 : 0);
    if (modes > 1) return fail("QK accumulation modes are mutually exclusive");
    if (cfg.qk_q_prescale <= 0.0f) return fail("Q prescale must be positive");

    const bool flush = cfg.o_accum_fp16 && cfg.o_accum_fp16_tile_flush;
    const bool fp16_acc = cfg.o_accum_fp16 && !flush;   // half accumulator, rescaled in place
    const float neg_inf = -std::numeric_limits<float>::infinity();
    const float scale = effective_scale(p);
    const int parts = cfg.kv_parallel_blocks;
    const int block_rows = std::min(cfg.br, p.seq_q);
    const size_t nstate = size_t(block_rows) * parts;          // state = part * block_rows + r
    const size_t stride = size_t(cfg.o_accum_np) * p.d_v;      // np accumulators per state
    std::vector<float> m(nstate), l(nstate), acc(nstate * stride), tile(stride), rebase(parts);
    std::vector<float> qprep(size_t(block_rows) * p.d_qk);
    std::vector<float> logit(std::min(cfg.bc, p.seq_kv));
    const bool prep = cfg.qk_scale_in_q || cfg.qk_q_prescale != 1.0f;
    const int shift = p.seq_kv - p.seq_q;                      // bottom-right causal offset

    for (int b = 0; b < p.batch; ++b) {
        for (int h = 0; h < p.n_head_q; ++h) {
            const size_t kv_base = (size_t(b) * p.n_head_kv + h / (p.n_head_q / p.n_head_kv)) * p.seq_kv;
            const size_t q_base = (size_t(b) * p.n_head_q + h) * p.seq_q;
            for (int ib = 0; ib < p.seq_q;) {
                const int nr = std::min(cfg.br, p.seq_q - ib);
                std::fill(m.begin(), m.end(), neg_inf);
                std::fill(l.begin(), l.end(), 0.0f);
                std::fill(acc.begin(), acc.end(), 0.0f);
                if (prep) {
                    // FP16 Q, optionally pre-scaled (attention_tiled_model.cpp:72-81)
                    for (int r = 0; r < nr; ++r) {
                        for (int d = 0; d < p.d_qk; ++d) {
                            float val = q[(q_base + ib + r) * p.d_qk + d];
                            val = fp16_round(cfg.qk_scale_in_q ? val * scale : val);
                            if (cfg.qk_q_prescale != 1.0f) val = fp16_round(val * cfg.qk_q_prescale);
                            qprep[size_t(r) * p.d_qk + d] = val;
                        }
                    }
                }
                for (int jb = 0; jb < p.seq_kv;) {
                    const int part = (jb / cfg.bc) % parts;
                    const int nc = std::min(cfg.bc, p.seq_kv - jb);
                    if (p.causal && jb > ib + nr - 1 + shift) break;   // no row of the block sees it
                    for (int r = 0; r < nr; ++r) {
                        const int i = ib + r;
                        if (p.causal && jb > i + shift) continue;
                        const size_t st = size_t(part) * block_rows + r;
                        const float* qrow = prep ? qprep.data() + size_t(r) * p.d_qk : q + (q_base + i) * p.d_qk;
                        float tmax = neg_inf;
                        for (int c = 0; c < nc; ++c) {
                            const int j = jb + c;
                            float x = neg_inf;
                            if (!p.causal || j <= i + shift) {
                                const float* key = k + (kv_base + j) * p.d_qk;
                                float dot = 0.0f;
                                if (cfg.qk_half2_chain > 0) {
                                    // even/odd half2 lanes flushed to FP32 every chain steps
                                    float lane0 = 0.0f, lane1 = 0.0f;
                                    int steps = 0;
                                    for (int d = 0; d < p.d_qk; d += 2) {
                                        lane0 = fp16_round_d(double(qrow[d]) * key[d] + lane0);
                                        if (d + 1 < p.d_qk) lane1 = fp16_round_d(double(qrow[d + 1]) * key[d + 1] + lane1);
                                        if (++steps == cfg.qk_half2_chain || d + 2 >= p.d_qk) {
                                            dot += lane0 + lane1;
                                            lane0 = lane1 = 0.0f;
                                            steps = 0;
                                        }
                                    }
                                } else {
                                    for (int d = 0; d < p.d_qk; ++d) {
                                        float prod = qrow[d] * key[d];
                                        if (cfg.qk_products_fp16) prod = fp16_round(prod);
                                        dot += prod;
                                        if (cfg.qk_accum_fp16 && ((d + 1) % 16 == 0 || d + 1 == p.d_qk)) dot = fp16_round(dot);
                                    }
                                }
                                dot /= cfg.qk_q_prescale;
                                x = cfg.qk_scale_in_q ? dot : dot * scale;
                                if (p.softcap > 0.0f) x = p.softcap * std::tanh(x / p.softcap);
                                if (mask) x += mask[size_t(i) * p.seq_kv + j];
                            }
                            logit[c] = x;
                            tmax = std::max(tmax, x);
                        }
                        const float m_new = std::max(m[st], tmax + cfg.kq_max_offset);
                        if (m_new == neg_inf) continue;
                        const float alpha = m[st] == neg_inf ? 0.0f : std::exp(m[st] - m_new);
                        float* racc = acc.data() + st * stride;
                        float tsum = 0.0f;
                        if (fp16_acc) {
                            const float half_alpha = fp16_round(alpha);
                            for (size_t d = 0; d < stride; ++d) racc[d] = fp16_round_d(double(racc[d]) * half_alpha);
                        } else {
                            std::fill(tile.begin(), tile.end(), 0.0f);
                            if (flush) for (size_t d = 0; d < stride; ++d) racc[d] *= alpha;
                        }
                        for (int c = 0; c < nc; ++c) {
                            float wgt = std::exp(logit[c] - m_new);
                            if (cfg.l_from_unrounded_p) tsum += wgt;
                            if (cfg.p_fp16) wgt = fp16_round(wgt);
                            if (!cfg.l_from_unrounded_p) tsum += wgt;
                            const size_t lane = size_t(c % cfg.o_accum_np) * p.d_v;
                            const float* val = v + (kv_base + jb + c) * p.d_v;
                            if (cfg.o_accum_fp16) {
                                float* dst = flush ? tile.data() : racc;
                                for (int d = 0; d < p.d_v; ++d)
                                    dst[lane + d] = fp16_round_d(double(wgt) * val[d] + dst[lane + d]);
                            } else {
                                for (int d = 0; d < p.d_v; ++d) tile[lane + d] += wgt * val[d];
                            }
                        }
                        if (flush) {
                            for (size_t d = 0; d < stride; ++d) racc[d] += tile[d];
                        } else if (!cfg.o_accum_fp16) {
                            for (size_t d = 0; d < stride; ++d) racc[d] = racc[d] * alpha + tile[d];
                        }
                        l[st] = l[st] * alpha + tsum;
                        m[st] = m_new;
                    }
                    jb += nc;
                }
                // Split-K combine (attention_tiled_model.cpp:183-222).
                for (int r = 0; r < nr; ++r) {
                    const size_t row = q_base + ib + r;
                    float gmax = neg_inf;
                    for (int part = 0; part < parts; ++part) {
                        const size_t st = size_t(part) * block_rows + r;
                        gmax = std::max(gmax, m[st]);
                        float* lanes = acc.data() + st * stride;
                        for (int ln = 1; ln < cfg.o_accum_np; ++ln) {
                            for (int d = 0; d < p.d_v; ++d) {
                                const float s = lanes[d] + lanes[size_t(ln) * p.d_v + d];
                                lanes[d] = fp16_acc ? fp16_round(s) : s;
                            }
                        }
                    }
                    float den = 0.0f;
                    for (int part = 0; part < parts; ++part) {
                        const size_t st = size_t(part) * block_rows + r;
                        rebase[part] = l[st] == 0.0f ? 0.0f : (parts == 1 ? 1.0f : std::exp(m[st] - gmax));
                        den += rebase[part] * l[st];
                    }
                    for (int d = 0; d < p.d_v; ++d) {
                        float num = 0.0f;
                        for (int part = 0; part < parts; ++part) {
                            const size_t st = size_t(part) * block_rows + r;
                            if (l[st] == 0.0f) continue;
                            num += rebase[part] * acc[st * stride + d];
                        }
                        if (parts == 1) num = acc[size_t(r) * stride + d];
                        float val = den == 0.0f ? 0.0f : num / den;
                        if (cfg.o_fp16_out) val = fp16_round(val);
                        o[row * p.d_v + d] = val;
                    }
                    if (lse) lse[row] = den == 0.0f ? neg_inf : gmax + std::log(den);
                }
                ib += nr;
            }
        }
    }
    return 0;
}

}  // extern "C"
