/*
 * p100/b200.h — C ABI of the B200 (sm_100a) decode hot path.
 *
 * This is the drop-in boundary for the quantised mat-vec, FlashAttention-vec
 * decode and tensor-parallel paths of Frostbite1536/P100.  Each entry point
 * names the reference interface it replaces.  Plain pointers, sizes and a
 * CUDA stream only: no C++ or PyTorch types cross this boundary, so the same
 * header serves C, C++ (include/p100/b200.hpp wraps it with exceptions),
 * ctypes, cgo or JNI callers.
 *
 * Conventions
 *   - The caller owns every device buffer.  All work is ordered on the given
 *     stream; no entry point synchronises the device or the stream.
 *   - Status codes never throw.  On failure p100_last_error() returns a
 *     thread-local description; shape errors use the reference's wording.
 *   - Entry points act on the calling thread's current device and leave it
 *     current.  They are thread-safe across distinct streams.
 *   - There is no CPU fallback.  Without an sm_100 device every compute entry
 *     point returns P100_ERR_UNSUPPORTED.
 *   - Every wait inside a kernel is bounded (about one second).  A wait that
 *     runs out sets a per-device flag that p100_device_error() reports as
 *     P100_ERR_TIMEOUT; the kernel returns instead of hanging.
 */
#ifndef P100_B200_H
#define P100_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Raised when a struct below changes layout: 2 added p100_attn_desc's
 * kv_type (p100_llama_config's kv_type followed within 2), 3
 * p100_llama_config's tensor_types.  A binding compares it with
 * p100_abi_version(). */
#define P100_B200_ABI_VERSION 3

typedef enum p100_status {
    P100_OK = 0,
    P100_ERR_INVALID = 1,      /* bad shape or argument (reference: std::invalid_argument)   */
    P100_ERR_CUDA = 2,         /* CUDA runtime error (reference: P100_CUDA_CHECK, check.h:7-17) */
    P100_ERR_NCCL = 3,         /* NCCL error in the tensor-parallel layer                     */
    P100_ERR_TIMEOUT = 4,      /* a bounded device-side wait ran out                          */
    P100_ERR_UNSUPPORTED = 5   /* no sm_100 device, or a shape this build does not handle     */
} p100_status;

/* Weight formats in the order of p100::qmv::Type (include/p100/qmv.h:20),
 * then ggml's Q5_K (176-byte) and Q6_K (210-byte) super-blocks of 256 values,
 * which the reference does not have (the Q4_K_M GGUF mix keeps some tensors
 * in them): p100_dequantize and p100_qmv only, on a general kernel. */
typedef enum p100_qtype { P100_Q4_0 = 0, P100_Q8_0 = 1, P100_Q4_K = 2, P100_Q5_K = 3, P100_Q6_K = 4 } p100_qtype;

/* K/V cache element types (llama.cpp's -ctk / -ctv f16, q8_0, q4_0, the
 * cache types the reference benchmarks: bench/phase0.sh:127).  A quantised
 * row of d values is d/32 ggml blocks along the head dimension: q8_0
 * {fp16 d, int8 q[32]} (34 bytes), q4_0 {fp16 d, u8 qs[16]} (18 bytes). */
typedef enum p100_kv_type { P100_KV_F16 = 0, P100_KV_Q8_0 = 1, P100_KV_Q4_0 = 2 } p100_kv_type;

/* Same type as cudaStream_t; 0 is the legacy default stream. */
typedef struct CUstream_st* p100_stream_t;
/* A tensor-parallel rank (see the tensor-parallel section). */
typedef struct p100_tp p100_tp;

/* ------------------------------------------------------------------ library */
int p100_abi_version(void);
/* Thread-local text of the last failure on this thread ("" after success). */
const char* p100_last_error(void);
const char* p100_status_name(p100_status status);
/* P100_OK if `device` is an sm_100 GPU this build has code for. */
p100_status p100_device_check(int device);
/* Reads, and with clear != 0 resets, the current device's error flag:
 * P100_ERR_TIMEOUT if a kernel gave up a bounded wait since the last clear,
 * P100_ERR_INVALID if a kernel read a device-resident token or position out
 * of range.  Synchronises the current device. */
p100_status p100_device_error(int clear);

/* --------------------------------------------------------- quantised mat-vec */
/* Elements and bytes per weight block (qmv_model.cpp:12-13); -1 if unknown. */
int p100_block_elems(int type);
int p100_block_bytes(int type);
/* Bytes of a rows x k matrix of `type` blocks, row-major along k. */
size_t p100_weight_bytes(int type, int rows, int k);
/* Bytes of batch rows of k activations in block_q8_1 layout: per 32 values
 * {fp16 d, fp16 sum, int8 q[32]} = 36 bytes. */
size_t p100_q8_1_bytes(int k, int batch);

/* Q8_1 activation quantisation; replaces p100::qmv::prepare's q8_1 fields
 * (include/p100/qmv.h:34, qmv_model.cpp:53-71) and llama.cpp's
 * quantize_row_q8_1.  x is batch rows of k fp32 (k % 32 == 0).  Bit-exact with
 * prepare(): d = fp16(max|x|/127), q = round-half-away(x/(max|x|/127)),
 * sum = fp16 of the XOR-butterfly sum of the original x. */
p100_status p100_q8_1_quantize(const float* x, void* x_q8_1, int k, int batch,
                               p100_stream_t stream);

/* Dequantise a rows x k weight matrix to fp32, out[r*k + i].  Bit-exact with
 * float(double(d)*sc*q - double(dmin)*mn) of qmv_model.cpp:143. */
p100_status p100_dequantize(int type, const void* w, int rows, int k, float* out,
                            p100_stream_t stream);

/* y[c*rows + r] = sum_i W[r][i] * x_c[i] for c < batch (1..16), the q81 path
 * of p100::qmv::evaluate (qmv_model.cpp:147-180) over whole matrices; the
 * device counterpart of llama.cpp's mul_mat_vec_q and of the reference's
 * prototype mmv_h2_<type>_b<B> (bench/micro/h2_mmv.cu:151-176, same output
 * layout).  w: rows x k blocks of `type` (2-byte alignment suffices; 16-byte
 * aligned rows take the bulk-copy path).  x_q8_1: p100_q8_1_bytes(k, batch).
 * Integer block dots are exact; FP32 accumulation order differs from the
 * sequential CPU model within 1e-3 * ||w|| * ||x||. */
p100_status p100_qmv(int type, const void* w, int rows, int k, const void* x_q8_1,
                     int batch, float* y, p100_stream_t stream);

/* Flags for p100_qmv_ex. */
#define P100_QMV_PDL 1u  /* launch as a programmatic dependent of the previous
                            kernel in the stream: weights are prefetched before
                            that kernel finishes, so they must not be written
                            by it.  Activations are read only after it ends. */
#define P100_QMV_TC 2u   /* batch 2..16 of Q4_0 / Q8_0 / Q4_K (16-byte aligned rows,
                            k % 256 == 0): the 5th-generation tensor-core kernel
                            (tcgen05.mma kind::i8, operands and accumulators in
                            tensor memory, weights by TMA) wherever it fits. */
#define P100_QMV_MMA 4u  /* batch 2..16: never the tcgen05 kernel (the mma.sync
                            kernel where it fits).  Without either flag, Q8_0 and
                            Q4_K matrices of rows x k >= 2^25 take the tcgen05
                            kernel (faster there: 1.2-1.5x on the Llama-3 FFN
                            shapes), everything else the mma.sync kernel.  The
                            two may not be combined. */
p100_status p100_qmv_ex(int type, const void* w, int rows, int k, const void* x_q8_1,
                        int batch, float* y, unsigned flags, p100_stream_t stream);
/* p100_q8_1_quantize with P100_QMV_PDL available: the quantiser launched as
 * a programmatic dependent of the previous kernel (it reads x after that
 * kernel ends), so its launch overlaps that kernel's tail. */
p100_status p100_q8_1_quantize_ex(const float* x, void* x_q8_1, int k, int batch, unsigned flags,
                                  p100_stream_t stream);
/* y = W . Q8_1(x) from fp32 activations x [batch][k], the bits of
 * p100_q8_1_quantize followed by p100_qmv_ex.  With x_q8_1
 * (p100_q8_1_bytes(k, batch)): the quantiser (flags apply to it) writes the
 * Q8_1 rows there and the mat-vec runs as its programmatic dependent.  With
 * x_q8_1 NULL: one launch, the quantisation inside the mat-vec (every CTA
 * quantises the row), at batch 1 on the team kernel only (16-byte aligned w
 * and x, rows of whole 16-byte units; else P100_ERR_UNSUPPORTED).  No
 * counterpart in the reference, whose callers quantise (prepare) before each
 * mat-vec. */
p100_status p100_qmv_f32(int type, const void* w, int rows, int k, const float* x, int batch,
                         void* x_q8_1, float* y, unsigned flags, p100_stream_t stream);

/* ---------------------------------------------------- h16 activation path */
/* The FP16-activation mat-vec, qmv::h16_model (qmv_model.cpp:53-71,92-133;
 * the reference's GPU prototype h16_prepass / mmv_h2_<type>,
 * bench/micro/h2_mmv.cu:99-176, with the same two-buffer layout).
 * p100_h16_prepare: x [batch][k] fp32 -> h [batch][k] fp16 (per 32-block
 * fp16(x / max|x|) in the 0,2,1,3 order of each group of four) and
 * ss [batch][k/32][2] fp32 {max|x|, butterfly sum of the rounded h}; the
 * same bits as qmv::prepare.  k % 32 == 0, ss 8-byte aligned. */
p100_status p100_h16_prepare(const float* x, void* h, float* ss, int k, int batch, p100_stream_t stream);
/* y[c*rows + r] = h16_model(row r, column c) with HFMA2 chains of `chain`
 * (8: the model's h8, 16: h16): each 32-block's value equals the model's bit
 * for bit; a row adds its blocks in order within each 128-column range and
 * the ranges by a fixed butterfly (k = 128: the model's row exactly).
 * k % 128 == 0 (Q4_K: % 256), k <= 32768, w and h 16-byte aligned. */
p100_status p100_qmv_h16(int type, const void* w, int rows, int k, const void* h, const float* ss, int batch,
                         int chain, float* y, p100_stream_t stream);

/* ---------------------------------------------------- FlashAttention decode */
/* AttnParams (include/p100/attention.h:27-41) plus the split and the strides of
 * a KV cache whose capacity exceeds seq_kv.  Layouts (attention.h:8-14):
 *   q   fp32 [batch][n_head_q][seq_q][d_qk]
 *   k   fp16 [batch][n_head_kv][seq_kv][d_qk]   (rows of kv_head_stride)
 *   v   fp16 [batch][n_head_kv][seq_kv][d_v]
 *   o   fp32 [batch][n_head_q][seq_q][d_v]
 *   lse fp32 [batch][n_head_q][seq_q]  (natural log; -inf for a fully masked row)
 *   mask fp32 [seq_q][seq_kv], additive, optional.
 * Query head h reads kv head h / (n_head_q / n_head_kv).
 * With kv_type q8_0 / q4_0, k and v hold the same rows as blocks (a row of
 * d values is d/32 blocks); strides still count values and must be
 * multiples of 64, and the kernel reads the blocks directly, with the
 * values dequantize_q8_0 / dequantize_q4_0 give (bench/micro/
 * dequant_nc.cu:32-48): the result equals p100_kv_to_f16 followed by the
 * fp16 decode bit for bit.  Quantised K/V need d 64 or 128 and 1, 2, 4 or 8
 * query heads per kv head. */
typedef struct p100_attn_desc {
    int batch, n_head_q, n_head_kv, seq_q, seq_kv, d_qk, d_v;
    float scale;      /* 0 means 1/sqrt(d_qk)          */
    float softcap;    /* 0 means off                   */
    int causal;       /* bottom-right alignment        */
    int kv_splits;    /* split-K parts per head, 0 = chosen for the device */
    long long kv_head_stride;   /* elements between kv heads, 0 = seq_kv * d */
    long long kv_batch_stride;  /* elements between batches,  0 = n_head_kv * head stride */
    int kv_type;      /* p100_kv_type of k and v; 0 = fp16 */
} p100_attn_desc;

/* validate (attention_reference.cpp:18-32): P100_OK, or P100_ERR_INVALID with
 * the reference's reason copied into why. */
p100_status p100_attn_validate(const p100_attn_desc* desc, char* why, size_t why_len);
/* Workspace bytes p100_fa_decode needs for desc on the current device. */
size_t p100_fa_workspace_size(const p100_attn_desc* desc);
/* Zero a workspace before its first use (the kernel leaves it zeroed). */
p100_status p100_fa_workspace_init(void* ws, size_t ws_bytes, p100_stream_t stream);
/* Split-K FlashAttention-vec decode; replaces attention_reference /
 * attention_tiled_model (attention_reference.cpp:87-135,
 * attention_tiled_model.cpp:52-227) and llama.cpp's FA VEC kernel with its
 * parallel_blocks combine.  seq_q == 1; d_qk == d_v in {64, 128, 256};
 * n_head_q / n_head_kv <= 8.  FP32 logits, online softmax and accumulation;
 * parts merged by the rebased combine of attention_tiled_model.cpp:183-222.
 * lse and mask may be NULL. */
p100_status p100_fa_decode(const p100_attn_desc* desc, const float* q, const void* k,
                           const void* v, const float* mask, float* o, float* lse,
                           void* ws, size_t ws_bytes, p100_stream_t stream);

/* The same decode without a caller-supplied workspace.  It has no counterpart
 * in the reference; it exists for callers that may not allocate device memory
 * at all: a host whose allocator owns the whole device budget, or a loop that
 * cannot afford the device-wide synchronisation a cudaMalloc/cudaFree implies.
 * The split-K partials live instead in a fixed P100_FA_STATIC_SCRATCH_BYTES
 * array inside the library, held on every GPU that loads the library until
 * the process exits.  Calls whose split needs more (p100_fa_workspace_size of
 * desc) are rejected with P100_ERR_INVALID; lower desc->kv_splits to fit.
 * The first call on a device looks up that device's copy of the array, so
 * make it before any stream capture.  All calls share one array: calls that
 * may run at the same time on the GPU (different streams, overlapping
 * launches) race and must be ordered by the caller.  Allocates nothing. */
#define P100_FA_STATIC_SCRATCH_BYTES (2u << 20)
p100_status p100_fa_decode_static(const p100_attn_desc* desc, const float* q, const void* k,
                                  const void* v, const float* mask, float* o, float* lse,
                                  p100_stream_t stream);

/* Quantised K/V view -> contiguous fp16: llama.cpp's ggml_get_to_fp16_nc_cuda
 * for q8_0 / q4_0 as FlashAttention's tile and MMA kernels call it before
 * every attention call, replacing dequantize_block and the reference's
 * dequantize_block_q_0_nc (bench/micro/dequant_nc.cu:53-121, patch 0002).
 * Value i00 of row i01 of plane (i02, i03) is value i00 % 32 of block
 * i03*s03 + i02*s02 + i01*s01 + i00/32 of src (strides in blocks, as ggml's
 * nb / type size); dst[((i03*ne02 + i02)*ne01 + i01)*ne00 + i00] =
 * fp16(float(q) * d) (q8_0) or fp16((float(nib) - 8) * d) (q4_0), nearest
 * even.  ne00 % 32 == 0, ne01 * ne00 / 8 < 2^31, src 2-byte and dst 16-byte
 * aligned. */
p100_status p100_kv_to_f16(int kv_type, const void* src, long long ne00, long long ne01, long long ne02,
                           long long ne03, long long s01, long long s02, long long s03, void* dst,
                           p100_stream_t stream);

/* ---------------------------------------------------- decode-step glue */
/* The reference stops at one mat-vec and one attention call; it has no decode
 * step, so these have no reference counterpart.  They follow Llama-3 as
 * llama.cpp runs it, with every floating-point operation in a fixed order
 * that the CPU restatement in oracle/ repeats, so each is bit-exact against
 * it.  All take device buffers and run on `stream`. */

/* x: batch rows of k fp32 (the residual stream).  If delta is not NULL,
 * x += delta first (written back to x).  Then
 * y = (x * (1 / sqrt(sum(x^2) / k + eps))) * w, quantised to Q8_1 into
 * x_q8_1 (p100_q8_1_bytes(k, batch)); y is also stored to y_out if not NULL.
 * k % 32 == 0. */
p100_status p100_rmsnorm_q8_1(float* x, const float* delta, const float* w, float eps, int k, int batch,
                              void* x_q8_1, float* y_out, p100_stream_t stream);

/* The decode step's RMSNorm fused into the batch-1 mat-vec that consumes it:
 * y[rows] = W * Q8_1(RMSNorm(x_in + delta) * norm_w), with x_in + delta also
 * stored to x_out (if not NULL; x_out must not alias x_in).  The Q8_1 row and
 * y equal p100_rmsnorm_q8_1 (x = x_in, delta) followed by p100_qmv bit for
 * bit; the row is built inside the mat-vec kernel while its weights stream
 * in, saving a launch.  k = 4096 or 8192, 16-byte aligned w, x_in, delta,
 * x_out and norm_w; other shapes return P100_ERR_UNSUPPORTED (use the two
 * calls).  flags as p100_qmv_ex.  No reference counterpart. */
p100_status p100_qmv_rmsnorm(int type, const void* w, int rows, int k, const float* x_in, const float* delta,
                             float* x_out, const float* norm_w, float eps, float* y, unsigned flags,
                             p100_stream_t stream);

/* Host: the RoPE table rope_cs[pos][i] = {cos, sin} of
 * pos * theta^(-2i/head_dim) (computed in double) for pos < max_pos. */
void p100_rope_table(float* rope_cs, int max_pos, int head_dim, float theta);

/* qkv: [n_head q | n_head_kv k | n_head_kv v] x head_dim fp32 (the fused QKV
 * mat-vec output).  At the device-resident position *pos_dev: rotates each
 * adjacent pair (2i, 2i+1) of the q and k heads by rope_cs[pos][i] (q in
 * place), and stores the rotated k and the v heads as fp16 (nearest) into
 * row pos of k_cache / v_cache, laid out [head][max_pos][head_dim] with
 * kv_head_stride elements between heads.  A position outside [0, max_pos)
 * writes nothing and sets the device flag (p100_device_error reports
 * P100_ERR_INVALID). */
p100_status p100_rope_kv_append(float* qkv, int n_head, int n_head_kv, int head_dim, const float* rope_cs,
                                int max_pos, const int* pos_dev, void* k_cache, void* v_cache,
                                long long kv_head_stride, p100_stream_t stream);

/* gate_up: batch rows of [gate (n) | up (n)] fp32.  h = silu(gate) * up with
 * silu(g) = g / (1 + exp(-g)), quantised to Q8_1 into x_q8_1.  n % 32 == 0. */
p100_status p100_swiglu_q8_1(const float* gate_up, int n, int batch, void* x_q8_1, p100_stream_t stream);

/* idx[b] (and val[b] if not NULL) = argmax of row b of x (n fp32): the lowest
 * index among equal maxima; NaN never wins. */
p100_status p100_argmax(const float* x, int n, int batch, int* idx, float* val, p100_stream_t stream);

/* One rank's reduce of the one-shot peer all-reduce, fused with RMSNorm +
 * Q8_1 (the graph decoder's exchange; no reference counterpart).  slots is
 * this rank's arena of [2][world][k] 64-bit words into which every rank's
 * push stores its partial sum, row i of rank r at [e & 1][r][i] as
 * (e << 32) | (the fp32 bits of the value), e = *epoch + 1.  The kernel
 * waits until every word it reads carries e — for at most wait_ns
 * nanoseconds (0: about a second) — then x += the world values added in
 * rank order, RMSNorm * w into x_q8_1 (p100_rmsnorm_q8_1's arithmetic), and
 * *epoch = e.  A wait that runs out raises P100_ERR_TIMEOUT in
 * p100_device_error() and the kernel returns normally (the sums then hold
 * whatever the slots held); the exchange state is then undefined.  k % 32 ==
 * 0, k <= 16384; x, w and slots 16-byte aligned. */
p100_status p100_peer_reduce_rmsnorm(float* x, const float* w, float eps, int k, void* x_q8_1, void* slots, int world,
                                     int rank, int* epoch, unsigned long long wait_ns, p100_stream_t stream);

/* --------------------------------------------------- batch-1 decoder */
/* A Llama-3-shaped model with synthetic weights, decoded one token per
 * p100_decoder_step.  No reference counterpart (see above).  Every linear
 * weight and the embedding use wtype; norms are fp32; the KV cache is fp16,
 * or q8_0 / q4_0 blocks with kv_type (head_dim 64 or 128 and 1, 2, 4 or 8
 * query heads per kv head: the new rows are quantised inside the attention
 * kernel, as ggml quantises them for a quantised cache).
 * With a tensor-parallel handle the decoder holds that rank's slices: q/k/v
 * and gate/up split by output rows, o and down along K with an NCCL
 * all-reduce after each, the LM head by vocabulary rows with an all-gather of
 * each rank's best candidate.  Position and token live on the device: a step
 * embeds *token, appends row *pos, attends over [0, *pos], writes the argmax
 * token and advances *pos, so steps chain without the host. */
typedef struct p100_llama_config {
    int n_layer, hidden, n_head, n_head_kv, head_dim, ffn, vocab, max_ctx;
    float rope_theta, norm_eps;
    int wtype;
    int flags;   /* P100_DEC_* (0: defaults) */
    int kv_type; /* p100_kv_type of the cache (0: fp16) */
    /* Per-tensor weight formats, or NULL for wtype everywhere: an array of
     * P100_DEC_TENSOR_TYPES(n_layer) p100_qtype values indexed by
     * P100_TT_EMBED, P100_TT_LM_HEAD and P100_TT_LAYER(layer, P100_TT_Q ..
     * P100_TT_DOWN), read during p100_decoder_create only.  llama.cpp's
     * Q4_K_M files, for one, keep attn_v, ffn_down and output in Q6_K in
     * some layers and Q4_K elsewhere.  A fused matrix (q|k|v, gate|up) then
     * holds each range's rows in its own format, one range after the other;
     * its mat-vec runs one launch per run of equal formats. */
    const int* tensor_types;
} p100_llama_config;
enum { P100_TT_EMBED = 0, P100_TT_LM_HEAD = 1 };
enum { P100_TT_Q = 0, P100_TT_K, P100_TT_V, P100_TT_O, P100_TT_GATE, P100_TT_UP, P100_TT_DOWN };
#define P100_TT_LAYER(layer, part) (2 + 7 * (layer) + (part))
#define P100_DEC_TENSOR_TYPES(n_layer) (2 + 7 * (n_layer))
/* Run each RMSNorm inside the mat-vec that consumes it (p100_qmv_rmsnorm;
 * hidden 4096 or 8192, no peer-memory all-reduce): the same bits with one
 * launch less per norm.  Off by default: on B200 at batch 1 it measured
 * slower (8B 579 against 604 tokens/s), because every block of the mat-vec
 * then repeats the norm after waiting for the previous kernel, where the
 * separate one-block norm kernel fits beside the previous mat-vec and starts
 * the moment it ends. */
#define P100_DEC_FUSED_NORM 1
/* Decode with the persistent step kernel (one cooperative launch a token,
 * see p100_decoder_path) where it applies, instead of the graph of separate
 * kernels.  Off by default: on B200 it measured slower than the graph
 * (Llama-3-8B shape at context 4096: 396 against 663 tokens/s on one GPU;
 * its grid barriers cost as much as the kernel boundaries they replace, and
 * its FP32 SIMT attention is latency-bound at eight warps per SM). */
#define P100_DEC_STEP 2
typedef struct p100_decoder p100_decoder;
/* Tensor ids (per layer where it applies). */
enum {
    P100_T_EMBED = 0,     /* [vocab][hidden] wtype (or its tensor type)     */
    P100_T_ATTN_NORM,     /* [hidden] fp32                                  */
    P100_T_WQKV,          /* rows [q heads | k heads | v heads] x hidden    */
    P100_T_WO,            /* [hidden] x (this rank's q heads * head_dim)    */
    P100_T_FFN_NORM,      /* [hidden] fp32                                  */
    P100_T_WGATE_UP,      /* rows [gate slice | up slice] x hidden          */
    P100_T_WDOWN,         /* [hidden] x (this rank's FFN slice)             */
    P100_T_OUT_NORM,      /* [hidden] fp32                                  */
    P100_T_LM_HEAD        /* this rank's vocabulary rows x hidden           */
};
/* Buffer ids. */
enum { P100_B_HIDDEN = 0, P100_B_LOGITS, P100_B_KCACHE, P100_B_VCACHE, P100_B_ROPE };
/* Allocates everything (weights, fp16 KV cache for max_ctx, scratch) on the
 * current device, or tp's device; tp may be NULL. */
p100_status p100_decoder_create(const p100_llama_config* cfg, p100_tp* tp, p100_decoder** out);
/* Synthetic weights from seed: block scales d = |N(0,1)| * 0.02 *
 * sqrt(256 / K) (K the unsplit matrix's input width, so activations keep
 * their scale at any width and depth), codes uniform, d divided per format
 * by 1 (Q4_0), 16 (Q8_0), 64 (Q4_K), 128 (Q5_K) or 256 (Q6_K) so that every
 * format's values have about the same RMS; norms uniform in [0.9, 1.1].
 * Every value is a function of (seed, tensor, global coordinates), so the
 * slices of a tensor-parallel rank equal the unsplit model's. */
p100_status p100_decoder_init_random(p100_decoder* d, unsigned long long seed);
/* KV rows [0, n_pos) of every layer: N(0,1) * scale as fp16. */
p100_status p100_decoder_fill_kv(p100_decoder* d, int n_pos, unsigned long long seed, float scale);
p100_status p100_decoder_set_state(p100_decoder* d, int pos, int token);
/* Synchronises the device, then reads the position and the last token.
 * Returns P100_ERR_TIMEOUT if a device-side wait ran out (the device flag of
 * p100_device_error, left set): the decoder must then be recreated. */
p100_status p100_decoder_state(p100_decoder* d, int* pos, int* token);
/* n_steps tokens on stream.  On the step path (p100_decoder_path) each token
 * is one cooperative launch of the persistent step kernel.  On the graph path
 * the first call captures one step as a CUDA graph (on a stream of its own,
 * so make it outside any capture) and every step replays it.  With tp, every
 * rank must call it the same number of times.  After a device-side wait ran
 * out (p100_device_error() == P100_ERR_TIMEOUT) the step path returns at once
 * from later launches: destroy and recreate the decoder. */
p100_status p100_decoder_step(p100_decoder* d, int n_steps, p100_stream_t stream);
/* Which kernels p100_decoder_step runs.  P100_DEC_PATH_STEP (with
 * P100_DEC_STEP in flags): the whole token
 * as one persistent kernel (one CTA per SM, phases meeting at grid barriers,
 * a producer warp streaming every weight matrix and K/V tile through a
 * shared-memory ring; the tensor-parallel all-reduce over NVLink peer memory
 * inside it).  It applies when every layer matrix and the LM head share one
 * of Q4_0, Q8_0 or Q4_K, the cache is fp16, head_dim is 64 or 128 with 1,
 * 2, 4 or 8 query heads per kv head, every
 * matrix's k is a multiple of 256, flags do not hold P100_DEC_FUSED_NORM,
 * and, with tp, every pair of ranks has peer access.  P100_DEC_PATH_GRAPH
 * (the default): one CUDA graph of separate kernels a token. */
enum { P100_DEC_PATH_GRAPH = 0, P100_DEC_PATH_STEP = 1 };
int p100_decoder_path(const p100_decoder* d);
/* Device address and size of a tensor or buffer (for tests and tools). */
p100_status p100_decoder_tensor(p100_decoder* d, int layer, int which, void** ptr, size_t* bytes, int* rows,
                                int* cols);
p100_status p100_decoder_buffer(p100_decoder* d, int which, void** ptr, size_t* bytes);
/* First vocabulary id of this rank's LM-head rows. */
int p100_decoder_vocab_offset(const p100_decoder* d);
/* Weight bytes one step streams on this rank (all layers' matrices + LM head). */
size_t p100_decoder_weight_bytes_per_token(const p100_decoder* d);
p100_status p100_decoder_destroy(p100_decoder* d);

/* ------------------------------------------------- tensor-parallel (NCCL) */
/* Row-split tensor parallelism over the GPUs of one box; replaces the
 * reference's two-GPU PCIe layer (src/p2p/p2p.cpp) for the per-layer
 * partial-sum exchange.  One handle per rank. */
#define P100_TP_ID_BYTES 128
/* A fresh communicator id (ncclGetUniqueId) for rank 0 to share. */
p100_status p100_tp_unique_id(void* id /* P100_TP_ID_BYTES */);
/* One rank of a multi-process group: binds `device` and joins the group. */
p100_status p100_tp_init_rank(const void* id, int nranks, int rank, int device, p100_tp** out);
/* All ranks of a single-process group (ncclCommInitAll): out[i] for devs[i]. */
p100_status p100_tp_create(int ngpu, const int* devs, p100_tp** out);
int p100_tp_rank(const p100_tp* tp);
int p100_tp_size(const p100_tp* tp);
int p100_tp_device(const p100_tp* tp);
/* In-place fp32 sum over ranks, ordered on stream (which belongs to the
 * rank's device).  In a group joined with p100_tp_init_rank whose GPUs all
 * have peer access to each other (the ranks agree while joining), counts up
 * to P100_TP_PEER_MAX run as one kernel over NVLink peer memory: every rank
 * gets the values added in rank order, the same bits on every rank; larger
 * counts, P100_TP_ALLREDUCE=nccl in the environment and p100_tp_create groups
 * use ncclAllReduce.  Every rank passes the same count (the path depends on
 * it).  A peer all-reduce waits up to 30 s for the other ranks (ranks may
 * reach it far apart, as with NCCL); a wait that runs out leaves buf
 * unchanged, raises P100_ERR_TIMEOUT in p100_device_error() and breaks the
 * group's peer path: later all-reduces return at once with the same flag. */
#define P100_TP_PEER_MAX 65536
p100_status p100_tp_allreduce_sum(p100_tp* tp, float* buf, size_t count, p100_stream_t stream);
/* 1 when this rank's all-reduces of up to P100_TP_PEER_MAX values run over
 * peer memory, else 0. */
int p100_tp_peer(const p100_tp* tp);
/* The same for every rank of a single-process group, as one NCCL group call. */
p100_status p100_tp_allreduce_sum_group(p100_tp* const* tps, int n, float* const* bufs,
                                        size_t count, const p100_stream_t* streams);
/* Gather `count` fp32 from each rank into out[rank*count ...] on every rank. */
p100_status p100_tp_allgather(p100_tp* tp, const float* in, float* out, size_t count,
                              p100_stream_t stream);
/* Aborts the communicator if it reports an asynchronous error; then frees it. */
p100_status p100_tp_destroy(p100_tp* tp);

/* ------------------------------------------------------ peer copies (p2p) */
/* C view of p100::p2p (include/p100/p2p.h of the reference, src/p2p/p2p.cpp),
 * which this library also exports with its C++ signatures. */
typedef struct p100_peer_link p100_peer_link;
enum { P100_PATH_PEER = 0, P100_PATH_STAGED = 1 };
/* Topology text as p100::p2p::describe(probe()); returns bytes needed. */
size_t p100_p2p_describe(char* out, size_t out_len);
int p100_p2p_disabled_by_env(void);
p100_status p100_peer_link_create(int src_dev, int dst_dev, size_t chunk_bytes, p100_peer_link** out);
int p100_peer_link_path(const p100_peer_link* link);
p100_status p100_peer_link_copy(p100_peer_link* link, void* dst, const void* src, size_t bytes,
                                p100_stream_t stream);
p100_status p100_peer_link_destroy(p100_peer_link* link);

#ifdef __cplusplus
}
#endif
#endif /* P100_B200_H */
