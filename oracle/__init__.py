"""CPU oracle for the p100_b200 hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg
import this package.  The product (``p100_b200``) never imports it.

Two ctypes-loaded libraries (built by ``oracle/Makefile``):

* ``lib/libp100_oracle.so`` — the restatement of the reference's CPU contract
  (``p100_oracle.cpp``), always available once built;
* ``_ref/libp100_ref.so`` — the reference's own ``src/reference/*.cpp``
  compiled where they lie, available where the reference sources were present
  at build time (``Ref.available()``).

The numpy-facing helpers below mirror ``p100::qmv::{prepare,evaluate}`` and
``p100::attention_{reference,tiled_model}`` (include/p100/qmv.h:17-49,
include/p100/attention.h:27-80).
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "lib" / "libp100_oracle.so"
REF_LIB = HERE / "_ref" / "libp100_ref.so"

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 4
TYPE_NAMES = {Q4_0: "q4_0", Q8_0: "q8_0", Q4_K: "q4_K"}   # the reference's types (its golden tables)
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}

# K/V cache element types (kv_oracle.cpp); a quantised row of d values holds
# d / 32 blocks of KV_BLOCK_BYTES.
KV_F16, KV_Q8_0, KV_Q4_0 = 0, 1, 2
KV_BLOCK_BYTES = {KV_Q8_0: 34, KV_Q4_0: 18}

# p100o_act / qmv::ActivationBlock: 68 four-byte fields.
ACT_DTYPE = np.dtype([("scale", "<f4"), ("sum", "<f4"), ("h", "<f4", (32,)),
                      ("qd", "<f4"), ("qsum", "<f4"), ("q", "<i4", (32,))])
assert ACT_DTYPE.itemsize == 272


class Attn(C.Structure):
    """AttnParams (include/p100/attention.h:27-41)."""
    _fields_ = [("batch", C.c_int), ("n_head_q", C.c_int), ("n_head_kv", C.c_int),
                ("seq_q", C.c_int), ("seq_kv", C.c_int), ("d_qk", C.c_int), ("d_v", C.c_int),
                ("scale", C.c_float), ("softcap", C.c_float), ("causal", C.c_int)]

    def __init__(self, batch=1, n_head_q=1, n_head_kv=1, seq_q=1, seq_kv=1, d_qk=128, d_v=128,
                 scale=0.0, softcap=0.0, causal=False):
        super().__init__(batch, n_head_q, n_head_kv, seq_q, seq_kv, d_qk, d_v, scale, softcap,
                         int(bool(causal)))

    def shapes(self):
        b, hq, hk, sq, sk = self.batch, self.n_head_q, self.n_head_kv, self.seq_q, self.seq_kv
        return ((b, hq, sq, self.d_qk), (b, hk, sk, self.d_qk), (b, hk, sk, self.d_v),
                (b, hq, sq, self.d_v), (b, hq, sq))


class Tiled(C.Structure):
    """TiledModelConfig (include/p100/attention.h:54-71), same defaults."""
    _fields_ = [("br", C.c_int), ("bc", C.c_int), ("qk_accum_fp16", C.c_int), ("p_fp16", C.c_int),
                ("o_fp16_out", C.c_int), ("qk_scale_in_q", C.c_int), ("qk_q_prescale", C.c_float),
                ("qk_products_fp16", C.c_int), ("qk_half2_chain", C.c_int),
                ("kq_max_offset", C.c_float), ("l_from_unrounded_p", C.c_int),
                ("o_accum_fp16", C.c_int), ("kv_parallel_blocks", C.c_int), ("o_accum_np", C.c_int),
                ("o_accum_fp16_tile_flush", C.c_int)]

    def __init__(self, br=64, bc=64, qk_accum_fp16=False, p_fp16=True, o_fp16_out=True, **kw):
        vals = dict(qk_scale_in_q=0, qk_q_prescale=1.0, qk_products_fp16=0, qk_half2_chain=0,
                    kq_max_offset=0.0, l_from_unrounded_p=0, o_accum_fp16=0, kv_parallel_blocks=1,
                    o_accum_np=1, o_accum_fp16_tile_flush=0)
        vals.update(kw)
        super().__init__(br, bc, int(qk_accum_fp16), int(p_fp16), int(o_fp16_out), **{
            k: (float(v) if k in ("qk_q_prescale", "kq_max_offset") else int(v)) for k, v in vals.items()})


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def build():
    """Compile the oracle (and, where the reference is present, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load(path, prefix):
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built; run make -C {HERE}")
    lib = C.CDLL(str(path))
    return lib


class _Base:
    prefix = ""

    def _f(self, name, restype, *argtypes):
        fn = getattr(self.lib, self.prefix + name)
        fn.restype = restype
        fn.argtypes = list(argtypes)
        return fn

    def _check(self, status):
        if status != 0:
            raise ValueError(self.last_error())
        return status


class Oracle(_Base):
    """The restated CPU contract (p100_oracle.cpp)."""
    prefix = "p100o_"

    def __init__(self, path=LIB):
        self.lib = _load(path, self.prefix)
        f = self._f
        vp, ip, fp = C.c_void_p, C.c_int, C.c_float
        self.last_error = lambda: f("last_error", C.c_char_p)().decode()
        self.fp16_round = f("fp16_round", fp, fp)
        self.fp16_round_d = f("fp16_round_d", fp, C.c_double)
        self.fp16_bits = f("fp16_bits", C.c_uint16, fp)
        self.fp16_value = f("fp16_value", fp, C.c_uint16)
        self._prepare = f("prepare", ip, vp, ip, vp)
        self._pack = f("pack_q8_1", None, vp, ip, vp)
        self._quantize = f("quantize_q8_1", ip, vp, ip, ip, vp)
        self._rng_new = f("rng_new", vp, C.c_uint32)
        self._rng_free = f("rng_free", None, vp)
        self._random_row = f("random_row", ip, ip, ip, vp, vp)
        self._dequantize = f("dequantize", ip, ip, vp, ip, ip, vp)
        self._evaluate = f("evaluate", ip, ip, vp, vp, ip, vp, vp)
        self._qmv = f("qmv_q81", ip, ip, vp, ip, ip, vp, ip, vp)
        self._qmv_h16 = f("qmv_h16", ip, ip, vp, ip, ip, vp, ip, ip, vp)
        self._qmv_mt = f("qmv_q81_threaded", C.c_double, ip, vp, ip, ip, vp, ip, vp, ip)
        self._validate = f("attn_validate", ip, vp, C.c_char_p, ip)
        self._attn_ref = f("attention_reference", ip, vp, vp, vp, vp, vp, vp, vp)
        self._attn_ref_mt = f("attention_reference_threaded", C.c_double, vp, vp, vp, vp, vp, vp, ip)
        self._attn_tiled = f("attention_tiled", ip, vp, vp, vp, vp, vp, vp, vp, vp)
        self._eff_scale = f("attn_effective_scale", fp, vp)
        self._fill_normal = f("fill_normal", None, C.c_uint32, fp, fp, ip, C.c_size_t, vp)
        self._fill_uniform = f("fill_uniform", None, C.c_uint32, fp, fp, ip, C.c_size_t, vp)
        self._rmsnorm = f("rmsnorm_q8_1", ip, vp, vp, vp, fp, ip, vp, vp)
        self._rope = f("rope_kv_append", ip, vp, ip, ip, ip, vp, ip, ip, vp, vp, C.c_longlong)
        self.dec_exp = f("dec_exp", fp, fp)
        self._swiglu = f("swiglu_q8_1", ip, vp, ip, vp)
        self._argmax = f("argmax", ip, vp, ip, vp)
        self._decode_step = f("decode_step", ip, vp, vp, vp, vp, vp, ip, ip, vp, vp)
        self._decode_step_kv = f("decode_step_kv", ip, vp, vp, ip, ip, vp, vp, vp, ip, ip, vp, vp)
        ll = C.c_int64
        self.kv_block_bytes = f("kv_block_bytes", ip, ip)
        self._kv_to_f16 = f("kv_to_f16", ip, ip, vp, ll, ll, ll, ll, ll, ll, ll, vp)
        self._kv_lcg = f("kv_lcg_blocks", None, ip, C.c_size_t, C.c_uint32, vp)
        self._kv_quantize = f("kv_quantize", ip, ip, vp, C.c_size_t, vp)

    # ------------------------------------------------------------ seeded inputs
    def fill_normal(self, seed, n, mean=0.0, stddev=1.0, round_fp16=False):
        out = np.zeros(n, dtype=np.float32)
        self._fill_normal(seed, mean, stddev, int(round_fp16), n, _ptr(out))
        return out

    def fill_uniform(self, seed, n, lo, hi, round_fp16=False):
        out = np.zeros(n, dtype=np.float32)
        self._fill_uniform(seed, lo, hi, int(round_fp16), n, _ptr(out))
        return out

    # ------------------------------------------------------------ quantised mat-vec
    def prepare(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size // 32, dtype=ACT_DTYPE)
        self._check(self._prepare(_ptr(x), x.size, _ptr(out)))
        return out

    def pack_q8_1(self, acts):
        out = np.zeros(acts.size * 36, dtype=np.uint8)
        self._pack(_ptr(acts), acts.size, _ptr(out))
        return out

    def quantize_q8_1(self, x, k):
        x = np.ascontiguousarray(x, dtype=np.float32)
        batch = x.size // k
        out = np.zeros(batch * (k // 32) * 36, dtype=np.uint8)
        self._check(self._quantize(_ptr(x), k, batch, _ptr(out)))
        return out

    def random_rows(self, type_, k, rows, seed):
        """rows weight rows from one generator seeded once (qmv_model.cpp:30-43)."""
        rb = k // BLOCK_ELEMS[type_] * BLOCK_BYTES[type_]
        out = np.zeros(rows * rb, dtype=np.uint8)
        rng = self._rng_new(seed)
        try:
            for r in range(rows):
                self._check(self._random_row(type_, k, rng, out[r * rb:].ctypes.data_as(C.c_void_p)))
        finally:
            self._rng_free(rng)
        return out

    def dequantize(self, type_, w, rows, k):
        out = np.zeros(rows * k, dtype=np.float32)
        self._check(self._dequantize(type_, _ptr(np.ascontiguousarray(w)), rows, k, _ptr(out)))
        return out.reshape(rows, k)

    def evaluate(self, type_, w_row, x, acts):
        """All paths of qmv::evaluate for one row: dict of exact/h16_exact/weight_norm/q81/h8/h16."""
        r = np.zeros(1, dtype=[("exact", "<f8"), ("h16_exact", "<f8"), ("weight_norm", "<f8"),
                               ("q81", "<f4"), ("h8", "<f4"), ("h16", "<f4")])
        x = np.ascontiguousarray(x, dtype=np.float32)
        self._check(self._evaluate(type_, _ptr(np.ascontiguousarray(w_row)), _ptr(x), x.size,
                                   _ptr(acts), _ptr(r)))
        return {n: r[n][0] for n in r.dtype.names}

    def qmv_q81(self, type_, w, rows, k, acts, batch):
        y = np.zeros(batch * rows, dtype=np.float32)
        self._check(self._qmv(type_, _ptr(np.ascontiguousarray(w)), rows, k, _ptr(acts), batch, _ptr(y)))
        return y.reshape(batch, rows)

    def qmv_h16(self, type_, w, rows, k, acts, batch, chain):
        """qmv::h16_model for every row and column (chain 8 = h8, 16 = h16)."""
        y = np.zeros(batch * rows, dtype=np.float32)
        self._check(self._qmv_h16(type_, _ptr(np.ascontiguousarray(w)), rows, k, _ptr(acts), batch, chain, _ptr(y)))
        return y.reshape(batch, rows)

    def qmv_q81_threaded(self, type_, w, rows, k, acts, batch, nthreads):
        y = np.zeros(batch * rows, dtype=np.float32)
        secs = self._qmv_mt(type_, _ptr(np.ascontiguousarray(w)), rows, k, _ptr(acts), batch, _ptr(y),
                            nthreads)
        if secs < 0:
            raise ValueError(self.last_error())
        return y.reshape(batch, rows), secs

    # ------------------------------------------------------------ attention
    def effective_scale(self, p):
        return self._eff_scale(C.byref(p))

    def validate(self, p):
        buf = C.create_string_buffer(256)
        ok = self._validate(C.byref(p), buf, 256)
        return bool(ok), buf.value.decode()

    def attention_reference(self, p, q, k, v, mask=None, want_lse=True):
        qs, ks, vs, os_, ls = p.shapes()
        o = np.zeros(os_, dtype=np.float32)
        lse = np.zeros(ls, dtype=np.float32) if want_lse else None
        args = [np.ascontiguousarray(a, dtype=np.float32) if a is not None else None for a in (q, k, v, mask)]
        self._check(self._attn_ref(C.byref(p), *[_ptr(a) for a in args], _ptr(o), _ptr(lse)))
        return o, lse

    def attention_reference_threaded(self, p, q, k, v, nthreads):
        qs, ks, vs, os_, ls = p.shapes()
        o = np.zeros(os_, dtype=np.float32)
        lse = np.zeros(ls, dtype=np.float32)
        args = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v)]
        secs = self._attn_ref_mt(C.byref(p), *[_ptr(a) for a in args], _ptr(o), _ptr(lse), nthreads)
        if secs < 0:
            raise ValueError(self.last_error())
        return o, lse, secs

    def attention_tiled(self, p, cfg, q, k, v, mask=None, want_lse=True):
        qs, ks, vs, os_, ls = p.shapes()
        o = np.zeros(os_, dtype=np.float32)
        lse = np.zeros(ls, dtype=np.float32) if want_lse else None
        args = [np.ascontiguousarray(a, dtype=np.float32) if a is not None else None for a in (q, k, v, mask)]
        self._check(self._attn_tiled(C.byref(p), C.byref(cfg), *[_ptr(a) for a in args], _ptr(o), _ptr(lse)))
        return o, lse


    # ------------------------------------------------------- decode-step glue
    def rmsnorm_q8_1(self, x, w, eps, delta=None):
        """Returns (x after x += delta, Q8_1 bytes, y) for one row (decode_oracle.cpp)."""
        x = np.array(x, dtype=np.float32, copy=True)
        k = x.size
        out = np.zeros(k // 32 * 36, dtype=np.uint8)
        y = np.zeros(k, dtype=np.float32)
        d = None if delta is None else np.ascontiguousarray(delta, dtype=np.float32)
        self._check(self._rmsnorm(_ptr(x), _ptr(d), _ptr(np.ascontiguousarray(w, dtype=np.float32)), eps, k,
                                  _ptr(out), _ptr(y)))
        return x, out, y

    def rope_kv_append(self, qkv, nq, nkv, hd, rope_cs, max_pos, pos, k_cache, v_cache, head_stride):
        """qkv rotated (copy); k_cache/v_cache (uint16 fp16 bits) updated in place."""
        qkv = np.array(qkv, dtype=np.float32, copy=True)
        self._check(self._rope(_ptr(qkv), nq, nkv, hd, _ptr(np.ascontiguousarray(rope_cs, dtype=np.float32)),
                               max_pos, pos, _ptr(k_cache), _ptr(v_cache), head_stride))
        return qkv

    def swiglu_q8_1(self, gate_up, n):
        out = np.zeros(n // 32 * 36, dtype=np.uint8)
        self._check(self._swiglu(_ptr(np.ascontiguousarray(gate_up, dtype=np.float32)), n, _ptr(out)))
        return out

    def argmax(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        val = np.zeros(1, dtype=np.float32)
        return self._argmax(_ptr(x), x.size, _ptr(val)), float(val[0])

    # ------------------------------------------------------ quantised K/V cache
    def kv_to_f16(self, kv_type, src, ne00, ne01, ne02=1, ne03=1, s01=None, s02=None, s03=None):
        """dequantize_block over a K/V view (dequant_nc.cu:53-121): fp16
        [ne03][ne02][ne01][ne00]; block strides default to a contiguous view."""
        nb = ne00 // 32
        s01 = nb if s01 is None else s01
        s02 = nb * ne01 if s02 is None else s02
        s03 = s02 * ne02 if s03 is None else s03
        src = np.ascontiguousarray(src, dtype=np.uint8)
        out = np.zeros((ne03, ne02, ne01, ne00), dtype=np.uint16)
        self._check(self._kv_to_f16(kv_type, _ptr(src), ne00, ne01, ne02, ne03, s01, s02, s03, _ptr(out)))
        return out.view(np.float16)

    def kv_lcg_blocks(self, kv_type, nblk, seed=12345):
        """nblk blocks from the reference's generator (dequant_nc.cu:144-149)."""
        out = np.zeros(nblk * KV_BLOCK_BYTES[kv_type], dtype=np.uint8)
        self._kv_lcg(kv_type, nblk, seed, _ptr(out))
        return out

    def kv_quantize(self, kv_type, x):
        """ggml's q8_0 / q4_0 block quantiser over x (size % 32 == 0): bytes."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.zeros(x.size // 32 * KV_BLOCK_BYTES[kv_type], dtype=np.uint8)
        self._check(self._kv_quantize(kv_type, _ptr(x), x.size, _ptr(out)))
        return out

    def decode_step(self, cfg, weights, k_cache, v_cache, rope_cs, pos, token, kv_type=KV_F16, append=True):
        """One token of the restated decoder.  cfg: LlamaConfig; weights: dict of
        host numpy arrays named as the decoder's tensors ('embed', 'attn_norm'
        [per layer], 'wqkv', 'wo', 'ffn_norm', 'wgu', 'wdown', 'out_norm',
        'lm_head').  Caches (uint16 fp16 bits, or uint8 q8_0 / q4_0 blocks with
        kv_type) are updated in place; append=False keeps a quantised cache's
        row pos as given.  Returns (next token, logits, final residual)."""
        L = cfg.n_layer
        keep = []

        def arr(a):
            a = np.ascontiguousarray(a)
            keep.append(a)
            return a.ctypes.data_as(C.c_void_p)

        def table(name):
            t = (C.c_void_p * L)(*[arr(a) for a in weights[name]])
            keep.append(t)
            return t

        w = LlamaWeights(arr(weights["embed"]), C.cast(table("attn_norm"), C.c_void_p),
                         C.cast(table("wqkv"), C.c_void_p), C.cast(table("wo"), C.c_void_p),
                         C.cast(table("ffn_norm"), C.c_void_p), C.cast(table("wgu"), C.c_void_p),
                         C.cast(table("wdown"), C.c_void_p), arr(weights["out_norm"]), arr(weights["lm_head"]))
        logits = np.zeros(cfg.vocab, dtype=np.float32)
        hidden = np.zeros(cfg.hidden, dtype=np.float32)
        tok = self._decode_step_kv(C.byref(cfg), C.byref(w), kv_type, int(bool(append)), _ptr(k_cache), _ptr(v_cache),
                                   _ptr(np.ascontiguousarray(rope_cs, dtype=np.float32)), pos, token, _ptr(logits),
                                   _ptr(hidden))
        if tok < 0:
            raise ValueError("decode_step rejected its arguments")
        return tok, logits, hidden


class LlamaConfig(C.Structure):
    """p100o_llama, the same fields as p100_llama_config."""
    _fields_ = [("n_layer", C.c_int), ("hidden", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("max_ctx", C.c_int),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("wtype", C.c_int),
                ("tensor_types", C.POINTER(C.c_int))]

    def __init__(self, *args, tensor_types=None, **kw):
        """tensor_types: None, or 2 + 7 * n_layer formats (embed, lm_head, then
        q k v o gate up down per layer), as the decoder's config takes them."""
        super().__init__(*args, **kw)
        self._tt = None
        if tensor_types is not None:
            self._tt = (C.c_int * len(tensor_types))(*[int(t) for t in tensor_types])
            self.tensor_types = C.cast(self._tt, C.POINTER(C.c_int))


class LlamaWeights(C.Structure):
    """p100o_llama_weights: host pointers (per-layer ones as pointer tables)."""
    _fields_ = [(n, C.c_void_p) for n in ("embed", "attn_norm", "wqkv", "wo", "ffn_norm", "wgu", "wdown",
                                          "out_norm", "lm_head")]


class Ref(_Base):
    """The reference's own CPU contract, compiled into oracle/_ref (ref_shim.cpp)."""
    prefix = "p100r_"

    @staticmethod
    def available():
        return REF_LIB.exists()

    def __init__(self, path=REF_LIB):
        self.lib = _load(path, self.prefix)
        f = self._f
        vp, ip, fp = C.c_void_p, C.c_int, C.c_float
        self.last_error = lambda: f("last_error", C.c_char_p)().decode()
        self.round_to_fp16 = f("round_to_fp16", fp, fp)
        self.round_to_fp16_d = f("round_to_fp16_d", fp, C.c_double)
        self.half_bits = f("half_bits", C.c_uint16, fp)
        self.half_value = f("half_value", fp, C.c_uint16)
        self._rng_new = f("rng_new", vp, C.c_uint32)
        self._rng_free = f("rng_free", None, vp)
        self._random_row = f("random_row", ip, ip, ip, vp, vp)
        self._prepare = f("prepare", ip, vp, ip, vp)
        self._evaluate = f("evaluate", ip, ip, vp, vp, ip, vp, vp, vp)
        self._validate = f("validate", ip, vp, C.c_char_p, ip)
        self._attn_ref = f("attention_reference", ip, vp, vp, vp, vp, vp, vp, vp)
        self._attn_tiled = f("attention_tiled", ip, vp, vp, vp, vp, vp, vp, vp, vp)
        self._eval_rows_mt = f("evaluate_rows_threaded", C.c_double, ip, vp, ip, ip, vp, vp, ip)

    def evaluate_rows_threaded(self, type_, w, rows, k, x, nthreads):
        """prepare(x) + evaluate() of every row on nthreads threads -> (q81 [rows], seconds)."""
        y = np.zeros(rows, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        secs = self._eval_rows_mt(type_, _ptr(np.ascontiguousarray(w)), rows, k, _ptr(x), _ptr(y), nthreads)
        if secs < 0:
            raise ValueError(self.last_error())
        return y, secs

    def random_rows(self, type_, k, rows, seed):
        rb = k // BLOCK_ELEMS[type_] * BLOCK_BYTES[type_]
        out = np.zeros(rows * rb, dtype=np.uint8)
        rng = self._rng_new(seed)
        try:
            for r in range(rows):
                self._check(self._random_row(type_, k, rng, out[r * rb:].ctypes.data_as(C.c_void_p)))
        finally:
            self._rng_free(rng)
        return out

    def prepare(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size // 32, dtype=ACT_DTYPE)
        self._check(self._prepare(_ptr(x), x.size, _ptr(out)))
        return out

    def evaluate(self, type_, w_row, x, acts):
        d3 = np.zeros(3, dtype=np.float64)
        f3 = np.zeros(3, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        self._check(self._evaluate(type_, _ptr(np.ascontiguousarray(w_row)), _ptr(x), x.size, _ptr(acts),
                                   _ptr(d3), _ptr(f3)))
        return dict(exact=d3[0], h16_exact=d3[1], weight_norm=d3[2], q81=f3[0], h8=f3[1], h16=f3[2])

    def validate(self, p):
        buf = C.create_string_buffer(256)
        ok = self._validate(C.byref(p), buf, 256)
        return bool(ok), buf.value.decode()

    def attention_reference(self, p, q, k, v, mask=None, want_lse=True):
        qs, ks, vs, os_, ls = p.shapes()
        o = np.zeros(os_, dtype=np.float32)
        lse = np.zeros(ls, dtype=np.float32) if want_lse else None
        args = [np.ascontiguousarray(a, dtype=np.float32) if a is not None else None for a in (q, k, v, mask)]
        self._check(self._attn_ref(C.byref(p), *[_ptr(a) for a in args], _ptr(o), _ptr(lse)))
        return o, lse

    def attention_tiled(self, p, cfg, q, k, v, mask=None, want_lse=True):
        qs, ks, vs, os_, ls = p.shapes()
        o = np.zeros(os_, dtype=np.float32)
        lse = np.zeros(ls, dtype=np.float32) if want_lse else None
        args = [np.ascontiguousarray(a, dtype=np.float32) if a is not None else None for a in (q, k, v, mask)]
        self._check(self._attn_tiled(C.byref(p), C.byref(cfg), *[_ptr(a) for a in args], _ptr(o), _ptr(lse)))
        return o, lse


_oracle = None


def oracle():
    """Process-wide Oracle instance (building the library on first use if needed)."""
    global _oracle
    if _oracle is None:
        if not LIB.exists():
            build()
        _oracle = Oracle()
    return _oracle


def host_cores():
    return len(os.sched_getaffinity(0))
