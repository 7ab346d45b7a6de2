// decoder.cuh — a batch-1 Llama-3-shaped decode step on one GPU or one rank
// of a tensor-parallel group, replayed as one CUDA graph per token.
//
// Included at the end of capi.cu (one translation unit): it drives the
// library's own mat-vec (run_qmv), attention (plan_fa/launch_fa_d) and glue
// kernels (decode.cuh).  The step per layer:
//   x += delta; xq = Q8_1(RMSNorm(x) * attn_norm)            rmsnorm_q8_1
//   qkv = Wqkv . xq                    (fused q|k|v rows)     team mat-vec
//   RoPE(q, k) at pos; k, v -> fp16 cache row pos;
//   attn = FA(q, K[0..pos], V[0..pos]) (length from device);
//   Q8_1(attn)                            one fa_mma_kernel (fused), or
//                                         rope_kv_append + FA + quantize
//   delta = Wo . Q8_1(attn)            (TP: all-reduce)       mat-vec
//   x += delta; xq = Q8_1(RMSNorm(x) * ffn_norm)
//   gu = Wgate_up . xq                 (fused gate|up rows)
//   delta = Wdown . Q8_1(silu(g) * u)  (TP: all-reduce)       swiglu_q8_1 + mat-vec
// then x += delta, RMSNorm, the LM head and argmax; argmax writes the next
// token and advances the position, both device-resident, so a step needs no
// host round trip and the captured graph is the same every token.
//
// Tensor parallelism (Megatron split, the row-split of BASELINE config 5):
// q/k/v and gate/up by output rows (heads, FFN slice), o and down along K
// (their inputs are local), the LM head by vocabulary rows; RMSNorm, the
// embedding and the residual stream are replicated.  Each rank initialises
// its slices from global coordinates, so TP=N holds the same model as TP=1.
#pragma once
#include "decode.cuh"
#include "step.cuh"

namespace p100b {
namespace {

struct DecTensor {
    uint8_t* ptr = nullptr;
    size_t bytes = 0;
    int rows = 0, cols = 0;   // cols in elements (weights) or 1 (vectors)
    // A weight matrix as runs of rows in one format each, stored one after
    // the other (q | k | v or gate | up ranges of equal format merged): part
    // p is prows[p] rows of ptype[p] at byte poff[p].
    int nparts = 0;
    int ptype[3] = {}, prows[3] = {};
    size_t poff[3] = {};
};

struct Decoder {
    p100_llama_config cfg{};
    p100_tp* tp = nullptr;
    int rank = 0, nranks = 1, device = 0, sms = 0;
    int nq = 0, nkv = 0, ffn = 0, vocab0 = 0, vocab_n = 0;   // this rank's slice
    std::vector<int> ttypes;                                 // P100_TT_* -> weight format
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    std::vector<DecTensor> attn_norm, wqkv, wo, ffn_norm, wgu, wdown;
    DecTensor embed, out_norm, lm_head;
    __half *kcache = nullptr, *vcache = nullptr;   // [layer][nkv][max_ctx][hd] (fp16, or blocks)
    size_t kv_row_bytes = 0;                       // one cache row: hd * 2, or hd/32 blocks
    float *x = nullptr, *delta = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *logits = nullptr;
    // P100_DEC_FUSED_NORM: the RMSNorms run inside the next mat-vec (team
    // kernel); the residual alternates between x2 and x, ending in x (2 per
    // layer + 1 swaps).
    bool fuse_norm = false;
    float* x2 = nullptr;
    float *rope = nullptr, *pair = nullptr, *cand = nullptr;
    uint8_t* xq = nullptr;
    int *pos = nullptr, *token = nullptr;
    uint8_t* fa_ws = nullptr;
    FaPlan fa_plan;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    // one-shot all-reduce over NVLink peer memory (tensor parallelism)
    bool peer_ar = false;
    uint8_t* ar_arena = nullptr;             // this rank's slots + flags
    void* ar_peer[dec::kArMaxRanks] = {};    // IPC mappings of the other ranks' arenas
    int* ar_epoch = nullptr;                 // completed-epoch counter (in the arena above)
    dec::PeerAr ar{};
    dec::PeerAr* ar_dev = nullptr;           // a device copy of ar (read by the push epilogue)
    // the persistent step kernel (step.cuh): one cooperative launch a token
    bool step_region = false;   // the arena holds its buffers (the config allows it)
    bool use_step = false;      // p100_decoder_step launches it
    uint8_t* st = nullptr;      // its buffers: layer table, attention partials, counters
    size_t st_layers = 0, st_ws_o = 0, st_ws_ml = 0, st_tickets = 0, st_cand = 0, st_ctr = 0;
    stp::Params sp{};
    size_t step_smem = 0;
    int step_type = 0;
};

size_t dec_weight_bytes(int type, int rows, int cols) {
    return size_t(rows) * (cols / elems_of(type)) * bytes_of(type);
}

template <typename... Exp, typename... Act>
p100_status launch_glue(void (*kern)(Exp...), dim3 grid, dim3 block, cudaStream_t s, const char* what,
                        Act&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, std::forward<Act>(args)...), what);
}

// The format of tensor id i (P100_TT_*).
int dec_ttype(const Decoder& d, int i) { return d.ttypes[size_t(i)]; }

const char* config_reason(const p100_llama_config& c, int nranks, const std::vector<int>& tt) {
    if (c.n_layer <= 0 || c.hidden <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
        c.vocab <= 0 || c.max_ctx <= 0)
        return "all model dimensions must be positive";
    if (tt.size() != size_t(P100_DEC_TENSOR_TYPES(c.n_layer))) return "n_layer above 2^20";
    if (!known_type(c.wtype)) return "unknown weight type";
    int blk = 1;
    for (int t : tt) {
        if (!known_type(t)) return "unknown weight type in tensor_types";
        blk = std::max(blk, elems_of(t));
    }
    if (c.flags & ~(P100_DEC_FUSED_NORM | P100_DEC_STEP)) return "unknown decoder flags";
    if (c.n_head % c.n_head_kv) return "n_head must be divisible by n_head_kv";
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) return "head_dim must be 64, 128 or 256";
    if (c.n_head / c.n_head_kv > 8) return "at most 8 query heads per kv head";
    if (c.kv_type != P100_KV_F16 && c.kv_type != P100_KV_Q8_0 && c.kv_type != P100_KV_Q4_0) return "unknown kv_type";
    if (c.kv_type != P100_KV_F16) {
        const int g = c.n_head / c.n_head_kv;
        if (c.head_dim == 256 || (g != 1 && g != 2 && g != 4 && g != 8))
            return "a quantised KV cache needs head_dim 64 or 128 and 1, 2, 4 or 8 query heads per kv head";
    }
    if (c.n_head % nranks || c.n_head_kv % nranks) return "heads must split evenly over the ranks";
    if (c.hidden % blk || c.hidden % 32) return "hidden must be whole weight blocks";
    if (c.hidden > dec::kNormMaxK) return "hidden above the RMSNorm kernel's limit (16384)";
    if ((c.n_head / nranks) * c.head_dim % blk) return "a rank's attention slice must be whole weight blocks";
    if (c.ffn % nranks || (c.ffn / nranks) % blk || (c.ffn / nranks) % 32)
        return "a rank's FFN slice must be whole weight blocks";
    if (c.vocab < nranks) return "vocab smaller than the number of ranks";
    if (!(c.norm_eps >= 0.0f) || !(c.rope_theta > 0.0f)) return "norm_eps must be >= 0 and rope_theta > 0";
    return nullptr;
}

// Whether the configuration suits the persistent step kernel: one weight
// format (Q4_0, Q8_0 or Q4_K) for every layer matrix and the LM head (the
// embedding may differ), an fp16 cache, head_dim 64 or 128, and matrices of
// whole 256-value groups (the team mat-vec).  Set in d.step_type.
bool dec_step_config_ok(Decoder& d) {
    const p100_llama_config& c = d.cfg;
    if (!(c.flags & P100_DEC_STEP) || (c.flags & P100_DEC_FUSED_NORM)) return false;
    if (c.kv_type != P100_KV_F16 || (c.head_dim != 64 && c.head_dim != 128)) return false;
    const int G = c.n_head / c.n_head_kv;
    if (d.nranks > stp::kMaxRanks || (G != 1 && G != 2 && G != 4 && G != 8)) return false;
    const int t = d.ttypes[P100_TT_LM_HEAD];
    if (t != P100_Q4_0 && t != P100_Q8_0 && t != P100_Q4_K) return false;
    for (size_t i = 0; i < d.ttypes.size(); ++i)
        if (i != P100_TT_EMBED && d.ttypes[i] != t) return false;
    if (c.hidden % 256 || (d.nq * c.head_dim) % 256 || d.ffn % 256) return false;
    d.step_type = t;
    return true;
}

p100_status dec_alloc(Decoder& d) {
    const p100_llama_config& c = d.cfg;
    const int hd = c.head_dim, L = c.n_layer;
    d.nq = c.n_head / d.nranks;
    d.nkv = c.n_head_kv / d.nranks;
    d.ffn = c.ffn / d.nranks;
    d.vocab0 = static_cast<int>(static_cast<long long>(c.vocab) * d.rank / d.nranks);
    d.vocab_n = static_cast<int>(static_cast<long long>(c.vocab) * (d.rank + 1) / d.nranks) - d.vocab0;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t at = off; off += align256(bytes); return at; };
    struct Req { DecTensor* t; size_t at; };
    std::vector<Req> reqs;
    auto tensor = [&](DecTensor& dt, int rows, int cols, size_t bytes) {
        dt.rows = rows;
        dt.cols = cols;
        dt.bytes = bytes;
        reqs.push_back({&dt, take(bytes)});
    };
    // a weight matrix of cols inputs from row ranges {format, rows}
    auto weight = [&](DecTensor& dt, int cols, std::initializer_list<std::pair<int, int>> ranges) {
        int rows = 0;
        size_t bytes = 0;
        dt.nparts = 0;
        for (const auto& r : ranges) {
            if (dt.nparts > 0 && dt.ptype[dt.nparts - 1] == r.first) {
                dt.prows[dt.nparts - 1] += r.second;
            } else {
                dt.ptype[dt.nparts] = r.first;
                dt.prows[dt.nparts] = r.second;
                dt.poff[dt.nparts] = bytes;
                ++dt.nparts;
            }
            rows += r.second;
            bytes += dec_weight_bytes(r.first, r.second, cols);
        }
        tensor(dt, rows, cols, bytes);
    };
    auto tt = [&](int l, int part) { return dec_ttype(d, P100_TT_LAYER(l, part)); };
    d.attn_norm.resize(L); d.wqkv.resize(L); d.wo.resize(L); d.ffn_norm.resize(L); d.wgu.resize(L); d.wdown.resize(L);
    for (int l = 0; l < L; ++l) {
        tensor(d.attn_norm[l], c.hidden, 1, size_t(c.hidden) * 4);
        weight(d.wqkv[l], c.hidden,
               {{tt(l, P100_TT_Q), d.nq * hd}, {tt(l, P100_TT_K), d.nkv * hd}, {tt(l, P100_TT_V), d.nkv * hd}});
        weight(d.wo[l], d.nq * hd, {{tt(l, P100_TT_O), c.hidden}});
        tensor(d.ffn_norm[l], c.hidden, 1, size_t(c.hidden) * 4);
        weight(d.wgu[l], c.hidden, {{tt(l, P100_TT_GATE), d.ffn}, {tt(l, P100_TT_UP), d.ffn}});
        weight(d.wdown[l], d.ffn, {{tt(l, P100_TT_DOWN), c.hidden}});
    }
    weight(d.embed, c.hidden, {{dec_ttype(d, P100_TT_EMBED), c.vocab}});
    tensor(d.out_norm, c.hidden, 1, size_t(c.hidden) * 4);
    weight(d.lm_head, c.hidden, {{dec_ttype(d, P100_TT_LM_HEAD), d.vocab_n}});
    d.kv_row_bytes = c.kv_type == P100_KV_Q8_0   ? size_t(hd / 32) * 34
                     : c.kv_type == P100_KV_Q4_0 ? size_t(hd / 32) * 18
                                                 : size_t(hd) * 2;
    const size_t kv_bytes = size_t(L) * d.nkv * c.max_ctx * d.kv_row_bytes;
    const size_t at_k = take(kv_bytes), at_v = take(kv_bytes);
    const int xq_k = std::max(c.hidden, std::max(d.nq * hd, d.ffn));
    const size_t at_x = take(size_t(c.hidden) * 4), at_delta = take(size_t(c.hidden) * 4);
    const size_t at_x2 = take(size_t(c.hidden) * 4);
    const size_t at_qkv = take(size_t(d.nq + 2 * d.nkv) * hd * 4), at_attn = take(size_t(d.nq) * hd * 4);
    const size_t at_gu = take(size_t(2) * d.ffn * 4), at_logits = take(size_t(d.vocab_n) * 4);
    const size_t at_rope = take(size_t(c.max_ctx) * (hd / 2) * 8);
    const size_t at_pair = take(8), at_cand = take(size_t(d.nranks) * 8);
    const size_t at_xq = take(size_t(xq_k / 32) * 36), at_pos = take(4), at_token = take(4);
    // attention over [0, max_ctx): split plan and its workspace
    p100_attn_desc ad = {};
    ad.batch = 1;
    ad.n_head_q = d.nq;
    ad.n_head_kv = d.nkv;
    ad.seq_q = 1;
    ad.seq_kv = c.max_ctx;
    ad.d_qk = ad.d_v = hd;
    ad.kv_head_stride = static_cast<long long>(c.max_ctx) * hd;
    ad.kv_type = c.kv_type;
    if (p100_status st = plan_fa(ad, d.sms, d.fa_plan)) return st;
    const size_t at_ws = take(std::max<size_t>(d.fa_plan.ws_total, 256));
    // the persistent step kernel's buffers, when the configuration allows it
    d.step_region = dec_step_config_ok(d);
    size_t at_st = 0;
    if (d.step_region) {
        const int G = c.n_head / c.n_head_kv;
        const size_t st0 = off;
        at_st = take(size_t(L) * sizeof(stp::Layer));
        d.st_ws_o = take(size_t(d.nkv) * stp::kMaxParts * G * hd * 4) - st0;
        d.st_ws_ml = take(size_t(d.nkv) * stp::kMaxParts * G * 8) - st0;
        d.st_tickets = take(size_t(d.nkv) * 4) - st0;
        d.st_cand = take(size_t(std::max(d.sms, 1)) * 8) - st0;
        d.st_ctr = take(256) - st0;   // grid barrier counter, two bases, abort word
        d.st_layers = 0;
    }
    d.arena_bytes = off;
    if (p100_status st = cuda_status(cudaMalloc(&d.arena, d.arena_bytes), "cudaMalloc(decoder)")) return st;
    for (const Req& r : reqs) r.t->ptr = d.arena + r.at;
    d.kcache = reinterpret_cast<__half*>(d.arena + at_k);
    d.vcache = reinterpret_cast<__half*>(d.arena + at_v);
    d.x = reinterpret_cast<float*>(d.arena + at_x);
    d.delta = reinterpret_cast<float*>(d.arena + at_delta);
    d.x2 = reinterpret_cast<float*>(d.arena + at_x2);
    d.qkv = reinterpret_cast<float*>(d.arena + at_qkv);
    d.attn = reinterpret_cast<float*>(d.arena + at_attn);
    d.gu = reinterpret_cast<float*>(d.arena + at_gu);
    d.logits = reinterpret_cast<float*>(d.arena + at_logits);
    d.rope = reinterpret_cast<float*>(d.arena + at_rope);
    d.pair = reinterpret_cast<float*>(d.arena + at_pair);
    d.cand = reinterpret_cast<float*>(d.arena + at_cand);
    d.xq = d.arena + at_xq;
    d.pos = reinterpret_cast<int*>(d.arena + at_pos);
    d.token = reinterpret_cast<int*>(d.arena + at_token);
    d.fa_ws = d.arena + at_ws;
    if (d.step_region) d.st = d.arena + at_st;
    if (p100_status st = cuda_status(cudaMemset(d.arena, 0, d.arena_bytes), "cudaMemset(decoder)")) return st;
    std::vector<float> table(size_t(c.max_ctx) * (hd / 2) * 2);
    p100_rope_table(table.data(), c.max_ctx, hd, c.rope_theta);
    return cuda_status(cudaMemcpy(d.rope, table.data(), table.size() * 4, cudaMemcpyHostToDevice), "copy rope table");
}

// Tensor ids mixed into the initialisation key (with the layer).
uint64_t dec_key(uint64_t seed, int layer, int id) {
    uint64_t z = seed ^ (uint64_t(layer + 1) << 32) ^ uint64_t(id + 1) * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 31)) * 0xd6e8feb86659fd93ull;
    return z ^ (z >> 32);
}

template <int T>
p100_status dec_init_w(uint8_t* w, size_t row_bytes, int rows, int blocks, uint64_t key, long long row0,
                       long long block0, float dscale) {
    const long long n = static_cast<long long>(rows) * blocks;
    if (n == 0) return P100_OK;
    dec::init_weights_kernel<T><<<unsigned((n + 255) / 256), 256>>>(w, row_bytes, rows, blocks, key, row0, block0,
                                                                      dscale);
    return launch_status("init_weights_kernel launch");
}

// Block scales |N(0,1)| * 0.02 * sqrt(256 / K), K the unsplit matrix's input
// width: the 0.02 of the mat-vec configs at K = 256, shrinking with fan-in so
// every projection's output keeps about the RMS of its input and the
// residual stream stays inside the fp16 fields of Q8_1 at any depth.
p100_status dec_init_matrix(int t, uint8_t* w, size_t row_bytes, int rows, int cols, uint64_t key, long long row0,
                            long long col0, int k_global) {
    const int blocks = cols / elems_of(t);
    const long long block0 = col0 / elems_of(t);
    const float dscale = 0.02f * std::sqrt(256.0f / float(k_global));
    switch (t) {
        case P100_Q4_0: return dec_init_w<P100_Q4_0>(w, row_bytes, rows, blocks, key, row0, block0, dscale);
        case P100_Q8_0: return dec_init_w<P100_Q8_0>(w, row_bytes, rows, blocks, key, row0, block0, dscale);
        case P100_Q4_K: return dec_init_w<P100_Q4_K>(w, row_bytes, rows, blocks, key, row0, block0, dscale);
        case P100_Q5_K: return dec_init_w<P100_Q5_K>(w, row_bytes, rows, blocks, key, row0, block0, dscale);
        default: return dec_init_w<P100_Q6_K>(w, row_bytes, rows, blocks, key, row0, block0, dscale);
    }
}

p100_status dec_init_vector(float* v, long long n, uint64_t key) {
    dec::init_uniform_kernel<<<unsigned((n + 255) / 256), 256>>>(v, n, key, 0, 0.9f, 1.1f);
    return launch_status("init_uniform_kernel launch");
}

// Every weight of this rank's slices.  Global coordinates: q rows of head h
// are h*hd.., k/v rows likewise per kv head; o and down columns are the K
// positions of this rank's heads / FFN slice; LM head rows are vocabulary ids.
p100_status dec_init_random(Decoder& d, uint64_t seed) {
    const p100_llama_config& c = d.cfg;
    const int hd = c.head_dim, H = c.hidden;
    enum { K_NORM1, K_Q, K_K, K_V, K_O, K_NORM2, K_GATE, K_UP, K_DOWN, K_EMB, K_NORM3, K_LM };
    // rows [row0, row0 + rows) of a range of format t stored at w
    auto range = [&](uint8_t* w, int t, int rows, int cols, uint64_t key, long long row0, long long col0,
                     int k_global) {
        return dec_init_matrix(t, w, dec_weight_bytes(t, 1, cols), rows, cols, key, row0, col0, k_global);
    };
    for (int l = 0; l < c.n_layer; ++l) {
        p100_status st = P100_OK;
        const int tq = dec_ttype(d, P100_TT_LAYER(l, P100_TT_Q)), tk = dec_ttype(d, P100_TT_LAYER(l, P100_TT_K));
        const int tv = dec_ttype(d, P100_TT_LAYER(l, P100_TT_V)), tg = dec_ttype(d, P100_TT_LAYER(l, P100_TT_GATE));
        uint8_t* w = d.wqkv[l].ptr;
        uint8_t* wk = w + dec_weight_bytes(tq, d.nq * hd, H);
        uint8_t* wv = wk + dec_weight_bytes(tk, d.nkv * hd, H);
        const long long q0 = static_cast<long long>(d.rank) * d.nq * hd, kv0 = static_cast<long long>(d.rank) * d.nkv * hd;
        const long long f0 = static_cast<long long>(d.rank) * d.ffn;
        if (!st) st = dec_init_vector(reinterpret_cast<float*>(d.attn_norm[l].ptr), H, dec_key(seed, l, K_NORM1));
        if (!st) st = range(w, tq, d.nq * hd, H, dec_key(seed, l, K_Q), q0, 0, H);
        if (!st) st = range(wk, tk, d.nkv * hd, H, dec_key(seed, l, K_K), kv0, 0, H);
        if (!st) st = range(wv, tv, d.nkv * hd, H, dec_key(seed, l, K_V), kv0, 0, H);
        if (!st) st = range(d.wo[l].ptr, d.wo[l].ptype[0], H, d.nq * hd, dec_key(seed, l, K_O), 0, q0, c.n_head * hd);
        if (!st) st = dec_init_vector(reinterpret_cast<float*>(d.ffn_norm[l].ptr), H, dec_key(seed, l, K_NORM2));
        if (!st) st = range(d.wgu[l].ptr, tg, d.ffn, H, dec_key(seed, l, K_GATE), f0, 0, H);
        if (!st) st = range(d.wgu[l].ptr + dec_weight_bytes(tg, d.ffn, H), dec_ttype(d, P100_TT_LAYER(l, P100_TT_UP)),
                            d.ffn, H, dec_key(seed, l, K_UP), f0, 0, H);
        if (!st) st = range(d.wdown[l].ptr, d.wdown[l].ptype[0], H, d.ffn, dec_key(seed, l, K_DOWN), 0, f0, c.ffn);
        if (st) return st;
    }
    p100_status st = range(d.embed.ptr, d.embed.ptype[0], c.vocab, H, dec_key(seed, -1, K_EMB), 0, 0, H);
    if (!st) st = dec_init_vector(reinterpret_cast<float*>(d.out_norm.ptr), H, dec_key(seed, -1, K_NORM3));
    if (!st) st = range(d.lm_head.ptr, d.lm_head.ptype[0], d.vocab_n, H, dec_key(seed, -1, K_LM), d.vocab0, 0, H);
    if (!st) st = cuda_status(cudaDeviceSynchronize(), "decoder initialisation");
    return st;
}

p100_status dec_fill_kv(Decoder& d, int npos, uint64_t seed, float scale) {
    const p100_llama_config& c = d.cfg;
    const int hd = c.head_dim;
    const long long hs = static_cast<long long>(c.max_ctx) * hd;
    const long long n = static_cast<long long>(d.nkv) * npos * hd;
    for (int l = 0; l < c.n_layer && n > 0; ++l) {
        const size_t layer_bytes = size_t(l) * d.nkv * c.max_ctx * d.kv_row_bytes;
        uint8_t* kl = reinterpret_cast<uint8_t*>(d.kcache) + layer_bytes;
        uint8_t* vl = reinterpret_cast<uint8_t*>(d.vcache) + layer_bytes;
        if (c.kv_type == P100_KV_F16) {
            const unsigned grid = unsigned((n + 255) / 256);
            dec::init_kv_kernel<<<grid, 256>>>(reinterpret_cast<__half*>(kl), d.nkv, npos, hd, hs,
                                               dec_key(seed, l, 100), d.rank * d.nkv, scale);
            dec::init_kv_kernel<<<grid, 256>>>(reinterpret_cast<__half*>(vl), d.nkv, npos, hd, hs,
                                               dec_key(seed, l, 101), d.rank * d.nkv, scale);
        } else {
            const unsigned grid = unsigned((n / 32 + 7) / 8);   // a warp per block
            auto kern = c.kv_type == P100_KV_Q8_0 ? dec::init_kv_quant_kernel<P100_KV_Q8_0>
                                                  : dec::init_kv_quant_kernel<P100_KV_Q4_0>;
            kern<<<grid, 256>>>(kl, d.nkv, npos, hd, c.max_ctx, dec_key(seed, l, 100), d.rank * d.nkv, scale);
            kern<<<grid, 256>>>(vl, d.nkv, npos, hd, c.max_ctx, dec_key(seed, l, 101), d.rank * d.nkv, scale);
        }
        if (p100_status st = launch_status("init_kv_kernel launch")) return st;
    }
    return cuda_status(cudaDeviceSynchronize(), "KV fill");
}

template <int T>
p100_status dec_embed_t(Decoder& d, cudaStream_t s) {
    const int slabs = d.cfg.hidden / 32;
    return launch_glue(dec::embed_kernel<T>, dim3((slabs + 255) / 256), dim3(256), s, "embed_kernel launch",
                       static_cast<const uint8_t*>(d.embed.ptr), dec_weight_bytes(T, 1, d.cfg.hidden), d.cfg.vocab,
                       d.cfg.hidden,
                       static_cast<const int*>(d.token), d.fuse_norm ? d.x2 : d.x);
}

// y = w . xq (k inputs), one mat-vec launch per part of w.
p100_status dec_qmv(const DecTensor& w, int k, const uint8_t* xq, float* y, cudaStream_t s) {
    int row = 0;
    for (int p = 0; p < w.nparts; ++p) {
        if (p100_status st = run_qmv(w.ptype[p], w.ptr + w.poff[p], w.prows[p], k, xq, 1, y + row, P100_QMV_PDL, s))
            return st;
        row += w.prows[p];
    }
    return P100_OK;
}

// x += delta (or, with peer_reduce, += the peer all-reduce of this epoch),
// then RMSNorm * w and Q8_1 into d.xq.
p100_status dec_rmsnorm(Decoder& d, const float* delta, const DecTensor& w, cudaStream_t s, bool peer_reduce = false) {
    dec::PeerAr ar{};
    if (peer_reduce) {
        ar = d.ar;
        delta = nullptr;
    }
    return launch_glue(dec::rmsnorm_q8_1_kernel, dim3(1), dim3(dec::kNormThreads), s, "rmsnorm_q8_1_kernel launch",
                       d.x, delta, reinterpret_cast<const float*>(w.ptr), d.cfg.norm_eps, d.cfg.hidden, d.xq,
                       static_cast<float*>(nullptr), ar);
}

// The row-parallel mat-vec delta = w . xq (k inputs) and its all-reduce.
// One rank: the mat-vec alone.  NCCL: the mat-vec, then an all-reduce of
// d.delta.  Peer memory: where the team kernel takes the matrix, its
// epilogue pushes the rows into every rank's slots (no separate kernel);
// else the mat-vec writes d.delta and ar_push_kernel pushes it.  The reduce
// runs in the next RMSNorm.
p100_status dec_qmv_allreduce(Decoder& d, const DecTensor& w, int k, cudaStream_t s) {
    if (d.peer_ar && w.nparts == 1) {
        p100_status st = P100_OK;
        if (run_qmv_push(w.ptype[0], w.ptr, w.prows[0], k, d.xq, d.ar_dev, d.ar, s, &st)) return st;
    }
    if (p100_status st = dec_qmv(w, k, d.xq, d.delta, s)) return st;
    if (!d.tp) return P100_OK;
    if (!d.peer_ar) return p100_tp_allreduce_sum(d.tp, d.delta, size_t(d.cfg.hidden), s);
    return launch_glue(dec::ar_push_kernel, dim3(dec::kArBlocks), dim3(256), s, "ar_push_kernel launch",
                       static_cast<const float*>(d.delta), d.ar);
}

// One token, recorded into stream s (a capture stream).
p100_status dec_record_step(Decoder& d, cudaStream_t s) {
    const p100_llama_config& c = d.cfg;
    const int hd = c.head_dim;
    const long long hs = static_cast<long long>(c.max_ctx) * hd;
    p100_status st = P100_OK;
    switch (d.embed.ptype[0]) {
        case P100_Q4_0: st = dec_embed_t<P100_Q4_0>(d, s); break;
        case P100_Q8_0: st = dec_embed_t<P100_Q8_0>(d, s); break;
        case P100_Q4_K: st = dec_embed_t<P100_Q4_K>(d, s); break;
        case P100_Q5_K: st = dec_embed_t<P100_Q5_K>(d, s); break;
        default: st = dec_embed_t<P100_Q6_K>(d, s); break;
    }
    // With the fused norms, cur is the residual stream and each norm writes
    // the updated stream to the other buffer.
    float* cur = d.fuse_norm ? d.x2 : d.x;
    auto norm_qmv = [&](const float* delta, const DecTensor& nw, const DecTensor& w, int rows, float* y) {
        if (!d.fuse_norm) {
            p100_status e = dec_rmsnorm(d, delta, nw, s, delta != nullptr && d.peer_ar);
            if (!e) e = dec_qmv(w, c.hidden, d.xq, y, s);
            return e;
        }
        float* next = cur == d.x ? d.x2 : d.x;
        const p100_status e = run_qmv_norm(w.ptype[0], w.ptr, rows, c.hidden, cur, delta, next,
                                           reinterpret_cast<const float*>(nw.ptr), c.norm_eps, y, P100_QMV_PDL, s);
        cur = next;
        return e;
    };
    for (int l = 0; l < c.n_layer && !st; ++l) {
        const size_t layer_bytes = size_t(l) * d.nkv * c.max_ctx * d.kv_row_bytes;
        const __half* kl = reinterpret_cast<const __half*>(reinterpret_cast<const uint8_t*>(d.kcache) + layer_bytes);
        const __half* vl = reinterpret_cast<const __half*>(reinterpret_cast<const uint8_t*>(d.vcache) + layer_bytes);
        st = norm_qmv(l == 0 ? nullptr : d.delta, d.attn_norm[l], d.wqkv[l], d.wqkv[l].rows, d.qkv);
        if (!st) {
            fa::Params prm = {};
            const FaPlan& plan = d.fa_plan;
            prm.q = d.qkv;
            prm.k = kl;
            prm.v = vl;
            prm.o = d.attn;
            prm.ws_o = plan.parts > 1 ? reinterpret_cast<float*>(d.fa_ws) : nullptr;
            prm.ws_ml = plan.parts > 1 ? reinterpret_cast<float*>(d.fa_ws + plan.ws_o) : nullptr;
            prm.tickets = plan.parts > 1 ? reinterpret_cast<unsigned*>(d.fa_ws + plan.ws_o + plan.ws_ml) : nullptr;
            prm.nkv = d.nkv;
            prm.G = plan.G;
            prm.seq = c.max_ctx;
            prm.parts = plan.parts;
            prm.nstage = plan.nstage;
            prm.head_stride = plan.head_stride;
            prm.batch_stride = plan.batch_stride;
            prm.scale = 1.0f / std::sqrt(float(hd));
            prm.softcap = 0.0f;
            prm.len_dev = d.pos;
            prm.len_add = 1;   // the row appended at pos is part of the context
            const bool fused = fa_use_mma(plan, prm);
            if (!fused && c.kv_type != P100_KV_F16) {
                st = set_error(P100_ERR_UNSUPPORTED, "a quantised KV cache needs the fused attention kernel");
                break;
            }
            if (fused) {
                // RoPE, the KV append and the Q8_1 of the output run inside
                // the attention kernel (fa::Params, fused decode step)
                prm.rope_cs = reinterpret_cast<const float2*>(d.rope);
                prm.nq_total = d.nq;
                prm.o_q81 = d.xq;
            } else {
                st = launch_glue(dec::rope_kv_append_kernel, dim3(d.nq + 2 * d.nkv), dim3(hd / 2), s,
                                 "rope_kv_append_kernel launch", d.qkv, d.nq, d.nkv, hd,
                                 reinterpret_cast<const float2*>(d.rope), c.max_ctx, static_cast<const int*>(d.pos),
                                 const_cast<__half*>(kl), const_cast<__half*>(vl), hs);
            }
            if (!st) {
                switch (hd) {
                    case 64: st = launch_fa_d<64>(plan, prm, d.nkv, s, true); break;
                    case 128: st = launch_fa_d<128>(plan, prm, d.nkv, s, true); break;
                    default: st = launch_fa_d<256>(plan, prm, d.nkv, s, true); break;
                }
            }
            if (!st && !fused) {
                const int k_o = d.nq * hd;
                st = launch_glue(q8_1_quantize_kernel, dim3((k_o / 32 + 7) / 8, 1), dim3(256), s,
                                 "q8_1_quantize_kernel launch", static_cast<const float*>(d.attn), d.xq, k_o, k_o / 32);
            }
        }
        if (!st) st = dec_qmv_allreduce(d, d.wo[l], d.nq * hd, s);
        if (!st) st = norm_qmv(d.delta, d.ffn_norm[l], d.wgu[l], 2 * d.ffn, d.gu);
        if (!st)
            st = launch_glue(dec::swiglu_q8_1_kernel, dim3((d.ffn / 32 + 7) / 8, 1), dim3(256), s,
                             "swiglu_q8_1_kernel launch", static_cast<const float*>(d.gu), d.ffn, d.xq);
        if (!st) st = dec_qmv_allreduce(d, d.wdown[l], d.ffn, s);
    }
    if (!st) st = norm_qmv(d.delta, d.out_norm, d.lm_head, d.vocab_n, d.logits);
    if (st) return st;
    if (!d.tp) {
        return launch_glue(dec::argmax_kernel, dim3(1), dim3(dec::kArgmaxThreads), s, "argmax_kernel launch",
                           static_cast<const float*>(d.logits), d.vocab_n, 0, static_cast<int*>(nullptr),
                           static_cast<float*>(nullptr), d.token, d.pos);
    }
    st = launch_glue(dec::argmax_pair_kernel, dim3(1), dim3(dec::kArgmaxThreads), s, "argmax_pair_kernel launch",
                     static_cast<const float*>(d.logits), d.vocab_n, d.vocab0, d.pair);
    if (!st) st = p100_tp_allgather(d.tp, d.pair, d.cand, 2, s);
    if (!st)
        st = launch_glue(dec::pick_candidates_kernel, dim3(1), dim3(32), s, "pick_candidates_kernel launch",
                         static_cast<const float*>(d.cand), d.nranks, d.token, d.pos);
    return st;
}

void dec_release_graph(Decoder& d) {
    if (d.graph_exec) cudaGraphExecDestroy(d.graph_exec);
    if (d.graph) cudaGraphDestroy(d.graph);
    d.graph_exec = nullptr;
    d.graph = nullptr;
}

p100_status dec_capture(Decoder& d) {
    cudaStream_t cs = nullptr;
    if (p100_status st = cuda_status(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "capture stream"))
        return st;
    p100_status st = cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    if (!st) {
        const p100_status rec = dec_record_step(d, cs);
        const std::string why = t_error;
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(cs, &g);
        if (rec) {
            if (g) cudaGraphDestroy(g);
            st = set_error(rec, "%s", why.c_str());
        } else if (e != cudaSuccess) {
            st = cuda_status(e, "end capture");
        } else {
            d.graph = g;
            st = cuda_status(cudaGraphInstantiate(&d.graph_exec, g, 0), "instantiate decode graph");
            if (st) dec_release_graph(d);
        }
    }
    cudaStreamDestroy(cs);
    return st;
}

// Device scratch of the create-time exchanges (a gather's input and output
// and an agreement word).  A static array, so every rank has it even where a
// local allocation failed and still enters every collective.
static __device__ float g_setup_scratch[16 + 16 * dec::kArMaxRanks + 4];

// The create-time exchanges of a tensor-parallel decoder.  Every rank calls
// every exchange, in the same order, whatever its local state: a local
// failure is carried into the next agreement (an all-reduce of failure
// counts) instead of skipping a collective, so no rank is ever left waiting
// in one.
struct SetupComm {
    Decoder& d;
    cudaStream_t s = nullptr;
    float* buf = nullptr;
    p100_status err = P100_OK;   // the first local error
    explicit SetupComm(Decoder& dd) : d(dd) {
        void* p = nullptr;
        note(cuda_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "setup stream"));
        note(cuda_status(cudaGetSymbolAddress(&p, g_setup_scratch), "setup scratch"));
        buf = static_cast<float*>(p);
    }
    ~SetupComm() {
        if (s) cudaStreamDestroy(s);
    }
    void note(p100_status st) {
        if (st && !err) err = st;
    }
    bool usable() const { return s && buf; }
    // every rank's `count` floats from `mine` into out (rank-major)
    void gather(const float* mine, int count, float* out) {
        const int world = d.nranks;
        if (usable()) {
            note(cuda_status(cudaMemcpyAsync(buf, mine, sizeof(float) * count, cudaMemcpyHostToDevice, s), "gather in"));
            note(p100_tp_allgather(d.tp, buf, buf + 16, size_t(count), s));
            note(cuda_status(cudaMemcpyAsync(out, buf + 16, sizeof(float) * count * world, cudaMemcpyDeviceToHost, s),
                             "gather out"));
            note(cuda_status(cudaStreamSynchronize(s), "gather sync"));
        } else {
            std::fill(out, out + size_t(count) * world, 0.f);
        }
    }
    // Agreement over the ranks (every rank gets the same): how many ranks
    // had a local error so far (errors) and how many passed ok = false.
    struct Votes {
        int errors = 0, declines = 0;
    };
    Votes agree(bool ok) {
        const float mine = (err ? 1000.f : 0.f) + (ok ? 0.f : 1.f);
        float all = 1000.f * d.nranks;
        if (usable()) {
            const int at = 16 + 16 * dec::kArMaxRanks;
            note(cuda_status(cudaMemcpyAsync(buf + at, &mine, sizeof(float), cudaMemcpyHostToDevice, s), "agree in"));
            note(p100_tp_allreduce_sum(d.tp, buf + at, 1, s));
            note(cuda_status(cudaMemcpyAsync(&all, buf + at, sizeof(float), cudaMemcpyDeviceToHost, s), "agree out"));
            note(cuda_status(cudaStreamSynchronize(s), "agree sync"));
        }
        const int v = static_cast<int>(all + 0.5f);
        return Votes{v / 1000, v % 1000};
    }
    // The status every rank returns after an agreement that saw errors.
    p100_status fail(const char* what) {
        if (err) return set_error(err, "%s: %s", what, t_error.c_str());
        return set_error(P100_ERR_CUDA, "%s: another rank failed", what);
    }
};

// Peer-memory exchange setup (tensor parallelism): every rank allocates an
// arena, the IPC handles go round an all-gather, and every rank maps the
// others'.  Used only if every pair of ranks' GPUs has peer access and
// P100_TP_ALLREDUCE is not "nccl", all ranks having agreed.  The arena holds
//   [2][world][hidden] 64-bit slots (the graph decoder's tagged words; the
//   step kernel uses their first half as fp32 slots of the same shape), then
//   in 256-byte cells: the graph decoder's epoch, the step kernel's argmax
//   candidates [world][2] and its 64-bit exchange counter, and a device copy
//   of this rank's exchange descriptor (read by the push epilogue).
// Collective: every rank calls it.  Returns an error only when the ranks
// agree that one of them failed; a declined or failed peer path leaves
// d.peer_ar false on every rank (NCCL carries the exchanges then).
p100_status dec_setup_peer_ar(Decoder& d) {
    const int world = d.nranks;
    if (!d.tp || world < 2 || world > dec::kArMaxRanks) return P100_OK;
    const char* mode = std::getenv("P100_TP_ALLREDUCE");
    const bool want = !(mode && std::strcmp(mode, "nccl") == 0);
    const int n = d.cfg.hidden;
    const bool shape_ok = n % (4 * dec::kArBlocks) == 0;   // the same on every rank
    SetupComm sc(d);
    // 1. (device, SM count) of every rank -> the verdict, agreed by all ranks
    std::vector<float> info(size_t(world) * 2);
    const float mine[2] = {float(d.device), float(d.sms)};
    sc.gather(mine, 2, info.data());
    bool ok = want && shape_ok;
    for (int r = 0; r < world && ok; ++r) {
        if (int(info[size_t(r) * 2 + 1]) != d.sms) ok = false;   // the step kernel's grids must match
        if (r == d.rank) continue;
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, d.device, int(info[size_t(r) * 2])) != cudaSuccess || !can) ok = false;
    }
    (void)cudaGetLastError();
    SetupComm::Votes v = sc.agree(ok);
    if (v.errors) return sc.fail("peer exchange setup");
    if (v.declines) return P100_OK;
    // 2. arenas and their IPC handles
    const size_t slot_bytes = size_t(2) * world * n * 8;
    const size_t arena_bytes = slot_bytes + 768 + 512;   // epoch | candidates | counter, 256 B each | descriptor
    cudaIpcMemHandle_t h{};
    p100_status st = cuda_status(cudaMalloc(&d.ar_arena, arena_bytes), "cudaMalloc(ar arena)");
    if (!st) st = cuda_status(cudaMemset(d.ar_arena, 0, arena_bytes), "cudaMemset(ar arena)");
    if (!st) st = cuda_status(cudaDeviceSynchronize(), "ar arena sync");
    if (!st) st = cuda_status(cudaIpcGetMemHandle(&h, d.ar_arena), "cudaIpcGetMemHandle");
    auto release = [&]() {
        for (int r = 0; r < dec::kArMaxRanks; ++r)
            if (d.ar_peer[r]) {
                cudaIpcCloseMemHandle(d.ar_peer[r]);
                d.ar_peer[r] = nullptr;
            }
        if (d.ar_arena) cudaFree(d.ar_arena);
        d.ar_arena = nullptr;
    };
    sc.note(st);
    v = sc.agree(true);
    if (v.errors) {
        release();
        return sc.fail("peer exchange setup");
    }
    // 3. every rank's handle; map the peers'
    std::vector<float> hmine(16), hall(size_t(world) * 16);
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    std::memcpy(hmine.data(), &h, 64);
    sc.gather(hmine.data(), 16, hall.data());
    st = sc.err;
    for (int r = 0; r < world && !st; ++r) {
        uint8_t* base = nullptr;
        if (r == d.rank) {
            base = d.ar_arena;
        } else {
            cudaIpcMemHandle_t hr;
            std::memcpy(&hr, hall.data() + size_t(r) * 16, 64);
            void* p = nullptr;
            st = cuda_status(cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
            d.ar_peer[r] = p;
            base = static_cast<uint8_t*>(p);
        }
        if (!st) {
            d.ar.slots[r] = reinterpret_cast<unsigned long long*>(base);
            d.sp.slots[r] = reinterpret_cast<float*>(base);
            d.sp.cslots[r] = reinterpret_cast<float*>(base + slot_bytes + 256);
            d.sp.xcount[r] = reinterpret_cast<unsigned long long*>(base + slot_bytes + 512);
        }
    }
    // the push epilogue reads this rank's exchange descriptor from device memory
    if (!st) {
        d.ar_epoch = reinterpret_cast<int*>(d.ar_arena + slot_bytes);
        d.ar.world = world;
        d.ar.rank = d.rank;
        d.ar.n = n;
        d.ar.epoch = d.ar_epoch;
        static_assert(sizeof(dec::PeerAr) <= 512, "PeerAr copy");
        d.ar_dev = reinterpret_cast<dec::PeerAr*>(d.ar_arena + slot_bytes + 768);
        st = cuda_status(cudaMemcpy(d.ar_dev, &d.ar, sizeof d.ar, cudaMemcpyHostToDevice), "copy exchange descriptor");
    }
    // 4. every rank's arena is zeroed and mapped before any rank pushes
    sc.note(st);
    v = sc.agree(true);
    if (v.errors) {
        release();
        return sc.fail("peer exchange setup");
    }
    d.peer_ar = true;
    return P100_OK;
}

// The step kernel for the decoder's format.
using StepKernel = void (*)(stp::Params);
StepKernel step_kernel_of(int type) {
    switch (type) {
        case P100_Q4_0: return stp::step_kernel<P100_Q4_0>;
        case P100_Q8_0: return stp::step_kernel<P100_Q8_0>;
        default: return stp::step_kernel<P100_Q4_K>;
    }
}

stp::Mat step_mat(const DecTensor& t, int type) {
    stp::Mat m;
    m.w = t.ptr;
    m.rows = t.rows;
    m.k = t.cols;
    m.row_bytes = static_cast<int>(dec_weight_bytes(type, 1, t.cols));
    m.ngroups = t.cols / 256;
    m.team = qmvt::team_lanes(m.ngroups);
    m.teams = stp::kCThreads / m.team;
    return m;
}

// Fills the step kernel's parameters and layer table and decides whether
// p100_decoder_step uses it: the arena holds its buffers, the device runs
// cooperative launches with one CTA of it per SM, and with several ranks the
// peer exchange is set up (every rank decides alike: same configuration,
// same verdict, same SM count).
p100_status dec_setup_step(Decoder& d) {
    d.use_step = false;
    if (!d.step_region || (d.nranks > 1 && !d.peer_ar)) return P100_OK;
    const p100_llama_config& c = d.cfg;
    const int T = d.step_type, hd = c.head_dim, L = c.n_layer;
    stp::Params& p = d.sp;
    std::vector<stp::Layer> layers(static_cast<size_t>(L));
    size_t stage_max = size_t(2) * stp::kTile * hd * 2;   // a K and a V tile
    int act_max = 0;
    bool whole_teams = true;   // every consumer lane in a whole team (see plan_team)
    auto note_mat = [&](const stp::Mat& m) {
        stage_max = std::max(stage_max, size_t(m.teams) * m.row_bytes);
        act_max = std::max(act_max, m.k / 32 * 36);
        if (m.team > stp::kCThreads || stp::kCThreads % m.team) whole_teams = false;
    };
    const size_t kv_layer = size_t(d.nkv) * c.max_ctx * hd;
    for (int l = 0; l < L; ++l) {
        stp::Layer& y = layers[size_t(l)];
        y.qkv = step_mat(d.wqkv[l], T);
        y.o = step_mat(d.wo[l], T);
        y.gu = step_mat(d.wgu[l], T);
        y.down = step_mat(d.wdown[l], T);
        y.attn_norm = reinterpret_cast<const float*>(d.attn_norm[l].ptr);
        y.ffn_norm = reinterpret_cast<const float*>(d.ffn_norm[l].ptr);
        y.kc = d.kcache + size_t(l) * kv_layer;
        y.vc = d.vcache + size_t(l) * kv_layer;
        for (const stp::Mat* m : {&y.qkv, &y.o, &y.gu, &y.down}) note_mat(*m);
    }
    p.lm = step_mat(d.lm_head, T);
    note_mat(p.lm);
    if (!whole_teams) return P100_OK;
    const size_t act_bytes = std::max<size_t>(size_t(act_max), size_t(stp::kAttnFloats) * 4);
    p.ring_off = static_cast<int>(stp::kActOff + round128(act_bytes));
    p.slot_bytes = static_cast<int>(round128(stage_max));
    p.nslot = std::min(stp::kMaxSlots, (stp::kSmemLimit - p.ring_off) / p.slot_bytes);
    if (p.nslot < 2) return P100_OK;
    d.step_smem = size_t(p.ring_off) + size_t(p.nslot) * p.slot_bytes;
    StepKernel kern = step_kernel_of(T);
    int coop = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, d.device) != cudaSuccess || !coop ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, stp::kSmemLimit) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, stp::kThreads, d.step_smem) != cudaSuccess ||
        per_sm < 1) {
        (void)cudaGetLastError();
        return P100_OK;
    }
    p.layers = reinterpret_cast<const stp::Layer*>(d.st + d.st_layers);
    p.n_layer = L;
    p.out_norm = reinterpret_cast<const float*>(d.out_norm.ptr);
    p.embed = d.embed.ptr;
    p.embed_type = d.embed.ptype[0];
    p.embed_row_bytes = dec_weight_bytes(p.embed_type, 1, c.hidden);
    p.hidden = c.hidden;
    p.nq = d.nq;
    p.nkv = d.nkv;
    p.G = c.n_head / c.n_head_kv;
    p.hd = hd;
    p.ffn = d.ffn;
    p.vocab = c.vocab;
    p.vocab0 = d.vocab0;
    p.max_ctx = c.max_ctx;
    p.eps = c.norm_eps;
    p.scale = 1.0f / std::sqrt(float(hd));
    p.rope = reinterpret_cast<const float2*>(d.rope);
    p.x0 = d.x2;
    p.x1 = d.x;
    p.delta = d.delta;
    p.qkv = d.qkv;
    p.attn_q81 = d.xq;
    p.gu = d.gu;
    p.ffn_q81 = d.xq;
    p.logits = d.logits;
    p.ws_o = reinterpret_cast<float*>(d.st + d.st_ws_o);
    p.ws_ml = reinterpret_cast<float*>(d.st + d.st_ws_ml);
    p.tickets = reinterpret_cast<unsigned*>(d.st + d.st_tickets);
    p.cand = reinterpret_cast<float*>(d.st + d.st_cand);
    p.bar = reinterpret_cast<unsigned long long*>(d.st + d.st_ctr);
    p.base = p.bar + 1;
    p.abort_flag = reinterpret_cast<int*>(d.st + d.st_ctr + 32);
    p.pos = d.pos;
    p.token = d.token;
    p.world = d.nranks;
    p.rank = d.rank;
    if (d.nranks == 1) {
        p.slots[0] = nullptr;
        p.cslots[0] = nullptr;
        p.xcount[0] = nullptr;
    }
    if (p100_status st = cuda_status(cudaMemcpy(d.st + d.st_layers, layers.data(), layers.size() * sizeof(stp::Layer),
                                                cudaMemcpyHostToDevice),
                                     "copy step layer table"))
        return st;
    d.use_step = true;
    return P100_OK;
}

// One token of the step kernel on stream s: a cooperative launch, one CTA per SM.
p100_status dec_launch_step(Decoder& d, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d.sms);
    cfg.blockDim = dim3(stp::kThreads);
    cfg.dynamicSmemBytes = d.step_smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, step_kernel_of(d.step_type), d.sp), "step_kernel launch");
}

// Collective: no rank unmaps or frees its arena before every rank's work is
// done (a peer's in-flight stores must never reach freed memory).
void dec_teardown_peer_ar(Decoder& d) {
    if (!d.ar_arena) return;
    if (d.tp) {
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        cudaDeviceSynchronize();
        p100_tp_allreduce_sum(d.tp, reinterpret_cast<float*>(d.ar_arena), 1, s);
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
    }
    for (int r = 0; r < dec::kArMaxRanks; ++r)
        if (d.ar_peer[r]) cudaIpcCloseMemHandle(d.ar_peer[r]);
    cudaFree(d.ar_arena);
    d.ar_arena = nullptr;
    d.peer_ar = false;
}

struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int dev) { cudaGetDevice(&prev); cudaSetDevice(dev); }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

}  // namespace
}  // namespace p100b

struct p100_decoder {
    p100b::Decoder d;
};

extern "C" {

void p100_rope_table(float* out, int max_pos, int head_dim, float theta) {
    const int half = head_dim / 2;
    for (int p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const double a = double(p) * std::pow(double(theta), -2.0 * i / double(head_dim));
            out[(size_t(p) * half + i) * 2] = float(std::cos(a));
            out[(size_t(p) * half + i) * 2 + 1] = float(std::sin(a));
        }
}

p100_status p100_rmsnorm_q8_1(float* x, const float* delta, const float* w, float eps, int k, int batch,
                              void* x_q8_1, float* y_out, p100_stream_t stream) {
    clear_error();
    if (k <= 0 || k % 32 || batch <= 0) return set_error(P100_ERR_INVALID, "k must be a positive multiple of 32");
    if (k > dec::kNormMaxK) return set_error(P100_ERR_UNSUPPORTED, "k above %d", dec::kNormMaxK);
    if (!x || !w || !x_q8_1) return set_error(P100_ERR_INVALID, "null buffer");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    dec::rmsnorm_q8_1_kernel<<<batch, dec::kNormThreads, 0, stream>>>(x, delta, w, eps, k,
                                                                        static_cast<uint8_t*>(x_q8_1), y_out,
                                                                        dec::PeerAr{});
    return launch_status("rmsnorm_q8_1_kernel launch");
}

p100_status p100_peer_reduce_rmsnorm(float* x, const float* w, float eps, int k, void* x_q8_1, void* slots, int world,
                                     int rank, int* epoch, unsigned long long wait_ns, p100_stream_t stream) {
    clear_error();
    if (k <= 0 || k % 32 || k % (4 * dec::kArBlocks)) return set_error(P100_ERR_INVALID, "k must be a positive multiple of 32");
    if (k > dec::kNormMaxK) return set_error(P100_ERR_UNSUPPORTED, "k above %d", dec::kNormMaxK);
    if (world < 1 || world > dec::kArMaxRanks || rank < 0 || rank >= world)
        return set_error(P100_ERR_INVALID, "rank %d of %d (at most %d ranks)", rank, world, dec::kArMaxRanks);
    if (!x || !w || !x_q8_1 || !slots || !epoch) return set_error(P100_ERR_INVALID, "null buffer");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16 ||
        reinterpret_cast<uintptr_t>(slots) % 16)
        return set_error(P100_ERR_INVALID, "x, w and slots must be 16-byte aligned");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    dec::PeerAr ar{};
    ar.slots[rank] = static_cast<unsigned long long*>(slots);
    ar.world = world;
    ar.rank = rank;
    ar.n = k;
    ar.epoch = epoch;
    ar.wait_ns = wait_ns;
    dec::rmsnorm_q8_1_kernel<<<1, dec::kNormThreads, 0, stream>>>(x, nullptr, w, eps, k, static_cast<uint8_t*>(x_q8_1),
                                                                    nullptr, ar);
    return launch_status("rmsnorm_q8_1_kernel launch");
}

p100_status p100_qmv_rmsnorm(int type, const void* w, int rows, int k, const float* x_in, const float* delta,
                             float* x_out, const float* norm_w, float eps, float* y, unsigned flags,
                             p100_stream_t stream) {
    clear_error();
    if (!known_type(type)) return set_error(P100_ERR_INVALID, "unknown weight type %d", type);
    if (rows < 0 || k <= 0 || k % elems_of(type)) return set_error(P100_ERR_INVALID, "whole weight blocks required");
    if (!w || !x_in || !norm_w || !y) return set_error(P100_ERR_INVALID, "null buffer");
    if (flags & ~P100_QMV_PDL) return set_error(P100_ERR_INVALID, "unknown flags 0x%x", flags);
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    if (rows == 0) return P100_OK;
    if (x_out == x_in) return set_error(P100_ERR_INVALID, "x_out must not alias x_in");
    const float* probe_out = x_out ? x_out : x_in + 4;   // alignment probe only when x_out is absent
    if (!qmv_norm_applies(type, w, rows, k, x_in, probe_out) || reinterpret_cast<uintptr_t>(delta) % 16 ||
        reinterpret_cast<uintptr_t>(norm_w) % 16)
        return set_error(P100_ERR_UNSUPPORTED, "fused RMSNorm mat-vec: k 4096 or 8192 and 16-byte aligned buffers");
    return run_qmv_norm(type, w, rows, k, x_in, delta, x_out, norm_w, eps, y, flags, stream);
}

p100_status p100_rope_kv_append(float* qkv, int n_head, int n_head_kv, int head_dim, const float* rope_cs,
                                int max_pos, const int* pos_dev, void* k_cache, void* v_cache,
                                long long kv_head_stride, p100_stream_t stream) {
    clear_error();
    if (n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 2048 || max_pos <= 0)
        return set_error(P100_ERR_INVALID, "bad RoPE shape");
    if (kv_head_stride < static_cast<long long>(max_pos) * head_dim)
        return set_error(P100_ERR_INVALID, "kv_head_stride must cover max_pos rows");
    if (!qkv || !rope_cs || !pos_dev || !k_cache || !v_cache) return set_error(P100_ERR_INVALID, "null buffer");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    dec::rope_kv_append_kernel<<<n_head + 2 * n_head_kv, head_dim / 2, 0, stream>>>(
        qkv, n_head, n_head_kv, head_dim, reinterpret_cast<const float2*>(rope_cs), max_pos, pos_dev,
        static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), kv_head_stride);
    return launch_status("rope_kv_append_kernel launch");
}

p100_status p100_swiglu_q8_1(const float* gate_up, int n, int batch, void* x_q8_1, p100_stream_t stream) {
    clear_error();
    if (n <= 0 || n % 32 || batch <= 0) return set_error(P100_ERR_INVALID, "n must be a positive multiple of 32");
    if (!gate_up || !x_q8_1) return set_error(P100_ERR_INVALID, "null buffer");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    dec::swiglu_q8_1_kernel<<<dim3((n / 32 + 7) / 8, batch), 256, 0, stream>>>(gate_up, n,
                                                                               static_cast<uint8_t*>(x_q8_1));
    return launch_status("swiglu_q8_1_kernel launch");
}

p100_status p100_argmax(const float* x, int n, int batch, int* idx, float* val, p100_stream_t stream) {
    clear_error();
    if (n <= 0 || batch <= 0) return set_error(P100_ERR_INVALID, "n and batch must be positive");
    if (!x || !idx) return set_error(P100_ERR_INVALID, "null buffer");
    if (p100_status st = require_sm100(nullptr, nullptr)) return st;
    dec::argmax_kernel<<<batch, dec::kArgmaxThreads, 0, stream>>>(x, n, 0, idx, val, nullptr, nullptr);
    return launch_status("argmax_kernel launch");
}

p100_status p100_decoder_create(const p100_llama_config* cfg, p100_tp* tp, p100_decoder** out) {
    clear_error();
    if (!cfg || !out) return set_error(P100_ERR_INVALID, "null argument");
    *out = nullptr;
    const int nranks = tp ? p100_tp_size(tp) : 1;
    std::vector<int> tt;
    if (cfg->n_layer > 0 && cfg->n_layer <= (1 << 20)) {
        tt.assign(size_t(P100_DEC_TENSOR_TYPES(cfg->n_layer)), cfg->wtype);
        if (cfg->tensor_types) tt.assign(cfg->tensor_types, cfg->tensor_types + tt.size());
    }
    if (const char* why = config_reason(*cfg, nranks, tt)) return set_error(P100_ERR_INVALID, "%s", why);
    int dev = 0;
    if (tp) {
        dev = p100_tp_device(tp);
    } else if (p100_status st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) {
        return st;
    }
    DeviceGuard guard(dev);
    int sms = 0;
    if (p100_status st = require_sm100(nullptr, &sms)) return st;
    auto* h = new p100_decoder();
    h->d.cfg = *cfg;
    h->d.cfg.tensor_types = nullptr;   // read here only: the caller's array need not outlive this call
    h->d.ttypes = std::move(tt);
    h->d.tp = tp;
    h->d.rank = tp ? p100_tp_rank(tp) : 0;
    h->d.nranks = nranks;
    h->d.device = dev;
    h->d.sms = sms;
    p100_status st = dec_alloc(h->d);
    if (tp) {
        // every rank learns whether every rank allocated before any rank
        // enters the exchanges below (a rank that returned here would leave
        // the others waiting in them)
        SetupComm sc(h->d);
        sc.note(st);
        if (sc.agree(true).errors) st = sc.fail("decoder allocation");
    }
    if (!st) st = dec_setup_peer_ar(h->d);
    if (!st) st = dec_setup_step(h->d);
    if (!st) {
        // P100_DEC_FUSED_NORM: RMSNorm inside the following mat-vec where
        // the team kernel has it (hidden 4096 or 8192); the one-shot peer
        // all-reduce keeps its reduce inside the separate RMSNorm kernel.
        Decoder& d = h->d;
        const int t = d.cfg.wtype, k = d.cfg.hidden;
        bool uniform = true;
        for (size_t i = 0; i < d.ttypes.size(); ++i)
            if (i != P100_TT_EMBED && d.ttypes[i] != t) uniform = false;
        d.fuse_norm = (d.cfg.flags & P100_DEC_FUSED_NORM) && uniform && !d.peer_ar &&
                      qmv_norm_applies(t, d.wqkv[0].ptr, d.wqkv[0].rows, k, d.x2, d.x) &&
                      qmv_norm_applies(t, d.wgu[0].ptr, 2 * d.ffn, k, d.x, d.x2) &&
                      qmv_norm_applies(t, d.lm_head.ptr, d.vocab_n, k, d.x2, d.x);
        clear_error();
    }
    if (st) {
        const std::string why = t_error;
        dec_teardown_peer_ar(h->d);
        if (h->d.arena) cudaFree(h->d.arena);
        delete h;
        return set_error(st, "%s", why.c_str());
    }
    *out = h;
    return P100_OK;
}

p100_status p100_decoder_init_random(p100_decoder* h, unsigned long long seed) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    DeviceGuard guard(h->d.device);
    return dec_init_random(h->d, seed);
}

p100_status p100_decoder_fill_kv(p100_decoder* h, int n_pos, unsigned long long seed, float scale) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    if (n_pos < 0 || n_pos > h->d.cfg.max_ctx) return set_error(P100_ERR_INVALID, "n_pos outside [0, max_ctx]");
    DeviceGuard guard(h->d.device);
    return dec_fill_kv(h->d, n_pos, seed, scale);
}

p100_status p100_decoder_set_state(p100_decoder* h, int pos, int token) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    if (pos < 0 || pos >= h->d.cfg.max_ctx) return set_error(P100_ERR_INVALID, "pos outside [0, max_ctx)");
    if (token < 0 || token >= h->d.cfg.vocab) return set_error(P100_ERR_INVALID, "token outside [0, vocab)");
    DeviceGuard guard(h->d.device);
    const int v[2] = {pos, token};
    p100_status st = cuda_status(cudaMemcpy(h->d.pos, &v[0], 4, cudaMemcpyHostToDevice), "set position");
    if (!st) st = cuda_status(cudaMemcpy(h->d.token, &v[1], 4, cudaMemcpyHostToDevice), "set token");
    return st;
}

p100_status p100_decoder_state(p100_decoder* h, int* pos, int* token) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    DeviceGuard guard(h->d.device);
    int v[2] = {0, 0};
    p100_status st = cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (!st) st = cuda_status(cudaMemcpy(&v[0], h->d.pos, 4, cudaMemcpyDeviceToHost), "read position");
    if (!st) st = cuda_status(cudaMemcpy(&v[1], h->d.token, 4, cudaMemcpyDeviceToHost), "read token");
    if (pos) *pos = v[0];
    if (token) *token = v[1];
    // a bounded wait that ran out (a peer that never pushed, say) leaves the
    // decode state undefined: report it here, where the loop synchronises
    int flag = 0;
    if (!st) st = cuda_status(cudaMemcpyFromSymbol(&flag, g_device_error, sizeof flag), "read device flag");
    if (!st && flag == kDevErrTimeout)
        st = set_error(P100_ERR_TIMEOUT, "a device-side wait ran out during a step; recreate the decoder");
    return st;
}

p100_status p100_decoder_step(p100_decoder* h, int n_steps, p100_stream_t stream) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    if (n_steps < 0) return set_error(P100_ERR_INVALID, "n_steps must be >= 0");
    DeviceGuard guard(h->d.device);
    if (h->d.use_step) {
        for (int i = 0; i < n_steps; ++i)
            if (p100_status st = dec_launch_step(h->d, stream)) return st;
        return P100_OK;
    }
    if (!h->d.graph_exec)
        if (p100_status st = dec_capture(h->d)) return st;
    for (int i = 0; i < n_steps; ++i)
        if (p100_status st = cuda_status(cudaGraphLaunch(h->d.graph_exec, stream), "launch decode graph")) return st;
    return P100_OK;
}

p100_status p100_decoder_tensor(p100_decoder* h, int layer, int which, void** ptr, size_t* bytes, int* rows,
                                int* cols) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    p100b::Decoder& d = h->d;
    const p100b::DecTensor* t = nullptr;
    const bool per_layer = which == P100_T_ATTN_NORM || which == P100_T_WQKV || which == P100_T_WO ||
                           which == P100_T_FFN_NORM || which == P100_T_WGATE_UP || which == P100_T_WDOWN;
    if (per_layer && (layer < 0 || layer >= d.cfg.n_layer)) return set_error(P100_ERR_INVALID, "layer out of range");
    switch (which) {
        case P100_T_EMBED: t = &d.embed; break;
        case P100_T_ATTN_NORM: t = &d.attn_norm[layer]; break;
        case P100_T_WQKV: t = &d.wqkv[layer]; break;
        case P100_T_WO: t = &d.wo[layer]; break;
        case P100_T_FFN_NORM: t = &d.ffn_norm[layer]; break;
        case P100_T_WGATE_UP: t = &d.wgu[layer]; break;
        case P100_T_WDOWN: t = &d.wdown[layer]; break;
        case P100_T_OUT_NORM: t = &d.out_norm; break;
        case P100_T_LM_HEAD: t = &d.lm_head; break;
        default: return set_error(P100_ERR_INVALID, "unknown tensor id %d", which);
    }
    if (ptr) *ptr = t->ptr;
    if (bytes) *bytes = t->bytes;
    if (rows) *rows = t->rows;
    if (cols) *cols = t->cols;
    return P100_OK;
}

p100_status p100_decoder_buffer(p100_decoder* h, int which, void** ptr, size_t* bytes) {
    clear_error();
    if (!h) return set_error(P100_ERR_INVALID, "null decoder");
    p100b::Decoder& d = h->d;
    const size_t kv = size_t(d.cfg.n_layer) * d.nkv * d.cfg.max_ctx * d.kv_row_bytes;
    void* p = nullptr;
    size_t n = 0;
    switch (which) {
        case P100_B_HIDDEN: p = d.x; n = size_t(d.cfg.hidden) * 4; break;
        case P100_B_LOGITS: p = d.logits; n = size_t(d.vocab_n) * 4; break;
        case P100_B_KCACHE: p = d.kcache; n = kv; break;
        case P100_B_VCACHE: p = d.vcache; n = kv; break;
        case P100_B_ROPE: p = d.rope; n = size_t(d.cfg.max_ctx) * d.cfg.head_dim * 4; break;
        default: return set_error(P100_ERR_INVALID, "unknown buffer id %d", which);
    }
    if (ptr) *ptr = p;
    if (bytes) *bytes = n;
    return P100_OK;
}

int p100_decoder_vocab_offset(const p100_decoder* h) { return h ? h->d.vocab0 : 0; }
int p100_decoder_path(const p100_decoder* h) {
    return h && h->d.use_step ? P100_DEC_PATH_STEP : P100_DEC_PATH_GRAPH;
}
size_t p100_decoder_weight_bytes_per_token(const p100_decoder* h) {
    if (!h) return 0;
    const p100b::Decoder& d = h->d;
    size_t n = d.lm_head.bytes;
    for (int l = 0; l < d.cfg.n_layer; ++l) n += d.wqkv[l].bytes + d.wo[l].bytes + d.wgu[l].bytes + d.wdown[l].bytes;
    return n;
}

p100_status p100_decoder_destroy(p100_decoder* h) {
    clear_error();
    if (!h) return P100_OK;
    DeviceGuard guard(h->d.device);
    p100b::dec_release_graph(h->d);
    p100b::dec_teardown_peer_ar(h->d);
    p100_status st = P100_OK;
    if (h->d.arena) st = cuda_status(cudaFree(h->d.arena), "cudaFree(decoder)");
    delete h;
    return st;
}

}  // extern "C"
