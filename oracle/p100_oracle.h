/*
 * p100_oracle.h — CPU restatement of the P100 numerics contract.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 decode
 * hot path: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load it.  The product library (p100_b200/lib/libp100_b200.so) never
 * links, loads or calls it, and has no CPU path of its own.
 *
 * Every function restates the arithmetic of the reference's CPU contract
 * (Frostbite1536/P100: the files under src/reference and include/p100) in the same
 * evaluation order, compiled with -O2 -ffp-contract=off as the reference is
 * (src/reference/CMakeLists.txt:6), so that results are bit-identical to it.
 * Each definition in p100_oracle.cpp cites the reference file:line it follows.
 *
 * Parity is pinned two ways (tests/test_oracle_*.py): against the reference
 * itself compiled from its own sources into oracle/_ref/ (oracle/Makefile),
 * and against the reference's committed golden outputs (the qmv-numerics
 * table, the tiled-model FNV digest, the analytic attention cases).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight formats, in the order of p100::qmv::Type (include/p100/qmv.h:20),
 * then ggml's Q5_K and Q6_K super-blocks (not in the reference's contract:
 * dequantisation and the q81 dot only; no h16 model). */
enum { P100O_Q4_0 = 0, P100O_Q8_0 = 1, P100O_Q4_K = 2, P100O_Q5_K = 3, P100O_Q6_K = 4 };

/* Thread-local description of the last failure (status -1). */
const char* p100o_last_error(void);

/* IEEE binary16 helpers (attention_reference.cpp:34-85,
 * attention_tiled_model.cpp:14-50, qmv_model.cpp:14-29). */
float    p100o_fp16_round(float x);
float    p100o_fp16_round_d(double x);
uint16_t p100o_fp16_bits(float x);
float    p100o_fp16_value(uint16_t h);

int p100o_block_elems(int type);
int p100o_block_bytes(int type);

/* The per-32 activation record of qmv::prepare (include/p100/qmv.h:28-34). */
typedef struct p100o_act {
    float scale, sum;   /* h16: max|x| and the butterfly sum of rounded x/scale */
    float h[32];        /* h16: fp16(x/scale), stored in the 0,2,1,3 lane order  */
    float qd, qsum;     /* q8_1: fp16(max|x|/127) and fp16(butterfly sum of x)  */
    int32_t q[32];      /* q8_1: round-half-away(x/d)                            */
} p100o_act;

/* qmv::prepare (qmv_model.cpp:53-71) for one activation row of k values. */
int p100o_prepare(const float* x, int k, p100o_act* out);
/* Pack prepared blocks into the 36-byte block_q8_1 wire layout used by the
 * GPU library: {fp16 d, fp16 sum, int8 q[32]}. */
void p100o_pack_q8_1(const p100o_act* a, int nblocks, void* out);
/* prepare + pack for batch rows of k values each. */
int p100o_quantize_q8_1(const float* x, int k, int batch, void* out);

/* One weight row of k values from the generator of qmv::random_row
 * (qmv_model.cpp:30-43).  rng_state is an opaque std::mt19937 created by
 * p100o_rng_new and advanced by each call. */
void* p100o_rng_new(uint32_t seed);
void  p100o_rng_free(void* rng);
int   p100o_random_row(int type, int k, void* rng, uint8_t* out);

/* Seeded inputs as the reference's tests draw them: n values from one
 * std::mt19937(seed) through std::normal_distribution<float>(mean, stddev) or
 * std::uniform_real_distribution<float>(lo, hi) (libstdc++), optionally
 * rounded to fp16 (tests/error_budget_split.cpp:101-112,
 * tests/test_tiled_model_flush.cpp:46-49). */
void p100o_fill_normal(uint32_t seed, float mean, float stddev, int round_fp16, size_t n, float* out);
void p100o_fill_uniform(uint32_t seed, float lo, float hi, int round_fp16, size_t n, float* out);

/* Dequantised weights, float(double(d)*sc*q - double(dmin)*mn), the value
 * qmv::evaluate forms at qmv_model.cpp:143. */
int p100o_dequantize(int type, const void* w, int rows, int k, float* out);

/* All paths of qmv::evaluate (qmv_model.cpp:134-185) for one weight row. */
typedef struct p100o_eval {
    double exact, h16_exact, weight_norm;
    float q81, h8, h16;
} p100o_eval;
int p100o_evaluate(int type, const void* w_row, const float* x, int k,
                   const p100o_act* acts, p100o_eval* out);

/* The h16 path only (qmv::h16_model, qmv_model.cpp:120-133, HFMA2 chain of
 * 8 or 16) for rows x batch outputs, y[c*rows + r]. */
int p100o_qmv_h16(int type, const void* w, int rows, int k, const p100o_act* acts, int batch, int chain, float* y);
/* The q81 path only (qmv_model.cpp:147-180) for rows x batch outputs,
 * y[c*rows + r]; acts holds batch rows of k/32 blocks. */
int p100o_qmv_q81(int type, const void* w, int rows, int k,
                  const p100o_act* acts, int batch, float* y);
/* Same, rows split over nthreads std::threads; returns wall seconds. */
double p100o_qmv_q81_threaded(int type, const void* w, int rows, int k,
                              const p100o_act* acts, int batch, float* y,
                              int nthreads);

/* AttnParams (include/p100/attention.h:27-41). */
typedef struct p100o_attn {
    int batch, n_head_q, n_head_kv, seq_q, seq_kv, d_qk, d_v;
    float scale, softcap;
    int causal;
} p100o_attn;

/* TiledModelConfig (include/p100/attention.h:54-71). */
typedef struct p100o_tiled {
    int br, bc;
    int qk_accum_fp16, p_fp16, o_fp16_out, qk_scale_in_q;
    float qk_q_prescale;
    int qk_products_fp16, qk_half2_chain;
    float kq_max_offset;
    int l_from_unrounded_p, o_accum_fp16, kv_parallel_blocks, o_accum_np;
    int o_accum_fp16_tile_flush;
} p100o_tiled;

float p100o_attn_effective_scale(const p100o_attn* p);
/* validate (attention_reference.cpp:18-32): 1 if valid; else 0 and the
 * reference's reason text in why. */
int p100o_attn_validate(const p100o_attn* p, char* why, int why_len);
/* attention_reference (attention_reference.cpp:87-135). */
int p100o_attention_reference(const p100o_attn* p, const float* q, const float* k,
                              const float* v, const float* mask, float* o, float* lse);
/* attention_tiled_model (attention_tiled_model.cpp:52-227). */
int p100o_attention_tiled(const p100o_attn* p, const p100o_tiled* cfg, const float* q,
                          const float* k, const float* v, const float* mask,
                          float* o, float* lse);
/* attention_reference with the query heads split over nthreads threads;
 * returns wall seconds (CPU baseline for the FA-vec decode kernel). */
double p100o_attention_reference_threaded(const p100o_attn* p, const float* q,
                                          const float* k, const float* v,
                                          float* o, float* lse, int nthreads);

/* ---- decode-step glue and one decode step (decode_oracle.cpp).  The
 * reference has no decode step: these restate the Llama-3 decode math in the
 * operation order of the GPU glue kernels (bit-exact targets) and chain the
 * pinned pieces above for a whole step (a tolerance target). */
int   p100o_rmsnorm_q8_1(float* x, const float* delta, const float* w, float eps, int k,
                         void* out_q81, float* y_out);
int   p100o_rope_kv_append(float* qkv, int nq, int nkv, int hd, const float* rope_cs, int max_pos,
                           int pos, uint16_t* k_cache, uint16_t* v_cache, long long head_stride);
float p100o_dec_exp(float x);
int   p100o_swiglu_q8_1(const float* gate_up, int n, void* out_q81);
/* Index of the largest value, lowest among equal ones; NaN never wins. */
int   p100o_argmax(const float* x, int n, float* val);

typedef struct p100o_llama {
    int n_layer, hidden, n_head, n_head_kv, head_dim, ffn, vocab, max_ctx;
    float rope_theta, norm_eps;
    int wtype;
    /* NULL, or per-tensor formats indexed as p100_llama_config's
     * tensor_types (embed, lm_head, then q k v o gate up down per layer);
     * fused matrices hold their ranges one after the other */
    const int* tensor_types;
} p100o_llama;
/* Host copies of the unsplit model, laid out as the GPU decoder's tensors. */
typedef struct p100o_llama_weights {
    const void* embed;
    const float* const* attn_norm;
    const void* const* wqkv;
    const void* const* wo;
    const float* const* ffn_norm;
    const void* const* wgu;
    const void* const* wdown;
    const float* out_norm;
    const void* lm_head;
} p100o_llama_weights;
/* One token at pos: appends row pos to the fp16 caches (as uint16 bits,
 * [layer][n_head_kv][max_ctx][head_dim]), writes vocab logits and the final
 * residual stream (hidden_out, optional), returns the argmax token (or -1). */
int p100o_decode_step(const p100o_llama* cfg, const p100o_llama_weights* w, uint16_t* k_cache,
                      uint16_t* v_cache, const float* rope_cs, int pos, int token, float* logits,
                      float* hidden_out);

/* ---- quantised K/V cache (kv_oracle.cpp) */
enum { P100O_KV_F16 = 0, P100O_KV_Q8_0 = 1, P100O_KV_Q4_0 = 2 };
/* p100o_decode_step over a cache of kv_type: fp16 bits as above, or q8_0 /
 * q4_0 blocks [layer][n_head_kv][max_ctx][head_dim/32]; the new rows are the
 * rotated k and the v of each kv head quantised by p100o_kv_quantize (append
 * = 1; with 0 a quantised cache's row pos is used as given), the attention
 * reads every row converted by p100o_kv_to_f16. */
int p100o_decode_step_kv(const p100o_llama* cfg, const p100o_llama_weights* w, int kv_type, int append,
                         void* k_cache, void* v_cache, const float* rope_cs, int pos, int token, float* logits,
                         float* hidden_out);
/* 34 (q8_0), 18 (q4_0), else 0. */
int p100o_kv_block_bytes(int kv_type);
/* dequantize_block over a K/V view (bench/micro/dequant_nc.cu:32-121):
 * dst[((i03*ne02 + i02)*ne01 + i01)*ne00 + i00] = fp16 bits of the value
 * i00 % 32 of block i03*s03 + i02*s02 + i01*s01 + i00/32. */
int p100o_kv_to_f16(int kv_type, const void* src, int64_t ne00, int64_t ne01, int64_t ne02, int64_t ne03,
                    int64_t s01, int64_t s02, int64_t s03, uint16_t* dst);
/* nblk blocks from the reference's LCG (dequant_nc.cu:144-149). */
void p100o_kv_lcg_blocks(int kv_type, size_t nblk, uint32_t seed, void* out);
/* ggml's q8_0 / q4_0 block quantisers over n values (n % 32 == 0). */
int p100o_kv_quantize(int kv_type, const float* x, size_t n, void* out);

#ifdef __cplusplus
}
#endif
