"""GGUF model files for the decoder: a reader, a writer, and a llama loader.

GGUF is ggml's model file (version 2 or 3): the magic "GGUF", a version, the
tensor and metadata counts, metadata as typed key/value pairs, one info
record per tensor (name, dimensions with the row length first, ggml type,
offset into the data section), then the data section at the file's
alignment (`general.alignment`, 32 by default).  Weight matrices are stored
row after row of quantised blocks, the layout `p100_qmv` reads, so a
tensor's bytes go to the GPU unchanged.

`load_llama` reads a llama-architecture file (the `llama.*` metadata keys
and `token_embd`, `blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output,
ffn_norm, ffn_gate, ffn_up, ffn_down}`, `output_norm`, `output` tensors, the
names llama.cpp writes) into a `Decoder`: q, k and v rows are stacked into
the decoder's fused QKV matrix and gate / up into its gate-up matrix, sliced
per rank under tensor parallelism.  llama.cpp stores q and k rows in the
order its RoPE of adjacent pairs expects, which is the decoder's RoPE, so no
rows are permuted.  Every matrix keeps its file format (Q4_0, Q8_0, Q4_K,
Q5_K or Q6_K, per tensor: a Q4_K_M file, for one, holds attn_v, ffn_down
and output in Q6_K in some layers), passed to the decoder as its
tensor_types; a tensor in any other format is rejected with its name.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"
# ggml tensor types (ggml.h enum ggml_type) and their (values, bytes) per block
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 2, 8, 12, 13, 14
GGML_BLOCKS = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34),
               GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}
GGML_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K",
              GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K"}
# ggml type -> p100_qtype
P100_TYPE = {GGML_Q4_0: 0, GGML_Q8_0: 1, GGML_Q4_K: 2, GGML_Q5_K: 3, GGML_Q6_K: 4}
GGML_OF_P100 = {v: k for k, v in P100_TYPE.items()}

# metadata value types
(T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64) = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


class GGUFError(ValueError):
    """A malformed file, or one the decoder cannot take."""


@dataclass
class TensorInfo:
    name: str
    dims: tuple          # row length first (ggml ne0, ne1, ...)
    ggml_type: int
    offset: int          # from the start of the data section

    @property
    def nbytes(self):
        if self.ggml_type not in GGML_BLOCKS:
            raise GGUFError(f"tensor {self.name}: ggml type {self.ggml_type} is not one this library reads")
        be, bb = GGML_BLOCKS[self.ggml_type]
        n = int(np.prod(self.dims, dtype=np.int64))
        if self.dims[0] % be:
            raise GGUFError(f"tensor {self.name}: rows of {self.dims[0]} values are not whole blocks")
        return n // be * bb


@dataclass
class GGUFFile:
    """A parsed GGUF file; tensor bytes are views into a read-only mapping."""
    path: str
    version: int = 0
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    data_offset: int = 0

    def __post_init__(self):
        self._f = open(self.path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:   # an empty file
            self._f.close()
            raise GGUFError(f"{self.path}: not a GGUF file") from e
        self._pos = 0
        self._parse()

    # ----------------------------------------------------------- parsing
    def _take(self, n):
        if self._pos + n > len(self._mm):
            raise GGUFError(f"{self.path}: truncated at byte {self._pos}")
        b = self._mm[self._pos:self._pos + n]
        self._pos += n
        return b

    def _scalar(self, t):
        fmt = _SCALAR[t]
        return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]

    def _string(self):
        n = self._scalar(T_U64)
        return self._take(n).decode("utf-8", errors="replace")

    def _value(self, t):
        if t in _SCALAR:
            return self._scalar(t)
        if t == T_STR:
            return self._string()
        if t == T_ARR:
            et, n = self._scalar(T_U32), self._scalar(T_U64)
            if et in _SCALAR and et != T_BOOL:
                fmt = _SCALAR[et]
                raw = self._take(n * struct.calcsize(fmt))
                return np.frombuffer(raw, dtype=np.dtype(fmt)).copy()
            return [self._value(et) for _ in range(n)]
        raise GGUFError(f"{self.path}: unknown metadata type {t} at byte {self._pos}")

    def _parse(self):
        if self._take(4) != GGUF_MAGIC:
            raise GGUFError(f"{self.path}: not a GGUF file")
        self.version = self._scalar(T_U32)
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} (2 and 3 are read)")
        n_tensors, n_kv = self._scalar(T_U64), self._scalar(T_U64)
        for _ in range(n_kv):
            key = self._string()
            self.metadata[key] = self._value(self._scalar(T_U32))
        for _ in range(n_tensors):
            name = self._string()
            nd = self._scalar(T_U32)
            dims = tuple(self._scalar(T_U64) for _ in range(nd))
            gt = self._scalar(T_U32)
            off = self._scalar(T_U64)
            self.tensors[name] = TensorInfo(name, dims, gt, off)
        align = int(self.metadata.get("general.alignment", 32))
        self.data_offset = (self._pos + align - 1) // align * align
        for t in self.tensors.values():
            if t.ggml_type in GGML_BLOCKS and self.data_offset + t.offset + t.nbytes > len(self._mm):
                raise GGUFError(f"{self.path}: tensor {t.name} runs past the end of the file")

    # ----------------------------------------------------------- access
    def tensor_bytes(self, name):
        """The raw bytes of a tensor (numpy uint8, a view into the file)."""
        if name not in self.tensors:
            raise GGUFError(f"{self.path}: no tensor {name}")
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=start)

    def close(self):
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:   # tensor views still alive: the mapping goes with the last of them
                pass
            self._f.close()
            self._mm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ----------------------------------------------------------------- writing
def _pack_value(v):
    """(type, bytes) of a metadata value: int -> u32 (i64 outside its range),
    float -> f32, str, bool, numpy 1-d arrays and lists of str."""
    if isinstance(v, bool):
        return T_BOOL, struct.pack("<?", v)
    if isinstance(v, (int, np.integer)):
        return (T_U32, struct.pack("<I", int(v))) if 0 <= int(v) < 2**32 else (T_I64, struct.pack("<q", int(v)))
    if isinstance(v, (float, np.floating)):
        return T_F32, struct.pack("<f", float(v))
    if isinstance(v, str):
        b = v.encode("utf-8")
        return T_STR, struct.pack("<Q", len(b)) + b
    if isinstance(v, np.ndarray):
        et = {np.dtype("<f4"): T_F32, np.dtype("<i4"): T_I32, np.dtype("<u4"): T_U32, np.dtype("<i8"): T_I64}[v.dtype]
        return T_ARR, struct.pack("<IQ", et, v.size) + v.tobytes()
    if isinstance(v, list) and all(isinstance(x, str) for x in v):
        body = b"".join(struct.pack("<Q", len(x.encode())) + x.encode() for x in v)
        return T_ARR, struct.pack("<IQ", T_STR, len(v)) + body
    raise TypeError(f"metadata value of type {type(v).__name__}")


def write_gguf(path, metadata, tensors, alignment=32):
    """Write a GGUF v3 file.  metadata: {key: value}; tensors: [(name, ggml
    type, dims with the row length first, bytes as a numpy array)]."""
    head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(metadata) + 1))
    meta = dict(metadata)
    meta["general.alignment"] = int(alignment)
    for k, v in meta.items():
        kb = k.encode("utf-8")
        t, body = _pack_value(v)
        head += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", t) + body
    off = 0
    blobs = []
    for name, gt, dims, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        info = TensorInfo(name, tuple(int(d) for d in dims), gt, off)
        if data.size != info.nbytes:
            raise GGUFError(f"tensor {name}: {data.size} bytes for dims {dims} of {GGML_NAMES.get(gt, gt)}")
        nb = name.encode("utf-8")
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", int(d)) for d in dims) + struct.pack("<IQ", gt, off)
        blobs.append((off, data))
        off = (off + data.size + alignment - 1) // alignment * alignment
    start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (start - len(head)))
        pos = 0
        for o, data in blobs:
            f.write(b"\0" * (o - pos))
            f.write(data.tobytes())
            pos = o + data.size


# ----------------------------------------------------------------- llama
def _meta(g, key, default=None):
    arch = g.metadata.get("general.architecture", "llama")
    full = f"{arch}.{key}"
    if full in g.metadata:
        return g.metadata[full]
    if default is None:
        raise GGUFError(f"{g.path}: metadata key {full} missing")
    return default


def llama_config(g, max_ctx=None, kv_type=0, flags=0):
    """The decoder configuration of a llama GGUF file: (LlamaConfig kwargs,
    the embedding's ggml type, whose format is the config's wtype)."""
    arch = g.metadata.get("general.architecture", "llama")
    if arch != "llama":
        raise GGUFError(f"{g.path}: architecture {arch!r} (llama is loaded)")
    hidden = int(_meta(g, "embedding_length"))
    n_head = int(_meta(g, "attention.head_count"))
    n_head_kv = int(_meta(g, "attention.head_count_kv", n_head))
    head_dim = int(_meta(g, "rope.dimension_count", hidden // n_head))
    if head_dim * n_head != hidden:
        raise GGUFError(f"{g.path}: head_dim {head_dim} x {n_head} heads is not the width {hidden}")
    emb = g.tensors.get("token_embd.weight")
    if emb is None:
        raise GGUFError(f"{g.path}: no tensor token_embd.weight")
    vocab = int(emb.dims[1])
    ctx = int(_meta(g, "context_length", 4096))
    wt = emb.ggml_type
    if wt not in P100_TYPE:
        raise GGUFError(f"{g.path}: token_embd.weight is {GGML_NAMES.get(wt, wt)}; the decoder reads "
                        + ", ".join(GGML_NAMES[t] for t in P100_TYPE))
    cfg = dict(n_layer=int(_meta(g, "block_count")), hidden=hidden, n_head=n_head, n_head_kv=n_head_kv,
               head_dim=head_dim, ffn=int(_meta(g, "feed_forward_length")), vocab=vocab,
               max_ctx=int(max_ctx or min(ctx, 4096)), rope_theta=float(_meta(g, "rope.freq_base", 10000.0)),
               norm_eps=float(_meta(g, "attention.layer_norm_rms_epsilon", 1e-5)), wtype=P100_TYPE[wt],
               flags=flags, kv_type=kv_type)
    return cfg, wt


def _check(g, name, gt, dims):
    """The bytes of tensor name after checking its dims and its format: gt, or
    any format the decoder's mat-vec reads when gt is None."""
    t = g.tensors.get(name)
    if t is None:
        raise GGUFError(f"{g.path}: no tensor {name}")
    if gt is None and t.ggml_type not in P100_TYPE:
        raise GGUFError(f"{g.path}: tensor {name} is {GGML_NAMES.get(t.ggml_type, t.ggml_type)}, the decoder "
                        "reads " + ", ".join(GGML_NAMES[x] for x in P100_TYPE))
    if gt is not None and t.ggml_type != gt:
        raise GGUFError(f"{g.path}: tensor {name} is {GGML_NAMES.get(t.ggml_type, t.ggml_type)}, "
                        f"the decoder needs {GGML_NAMES.get(gt, gt)}")
    if tuple(t.dims) != tuple(dims):
        raise GGUFError(f"{g.path}: tensor {name} has dims {t.dims}, expected {tuple(dims)}")
    return g.tensor_bytes(name)


# Per-layer matrices in the order of the decoder's tensor_types (P100_TT_Q .. P100_TT_DOWN).
LAYER_MATRICES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def llama_tensors(g, cfg):
    """Check every tensor the decoder reads (name, format, dims) before any
    device work; returns the name of the LM head tensor (`output.weight`, or
    `token_embd.weight` when the two are tied) and the tensor_types list
    (p100 formats: embedding, LM head, then each layer's LAYER_MATRICES)."""
    H, hd, F, V = cfg["hidden"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]
    nq, nkv = cfg["n_head"], cfg["n_head_kv"]
    lm = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    need = [("token_embd.weight", None, (H, V)), (lm, None, (H, V)), ("output_norm.weight", GGML_F32, (H,))]
    dims = {"attn_q": (H, nq * hd), "attn_k": (H, nkv * hd), "attn_v": (H, nkv * hd), "attn_output": (nq * hd, H),
            "ffn_gate": (H, F), "ffn_up": (H, F), "ffn_down": (F, H)}
    for l in range(cfg["n_layer"]):
        b = f"blk.{l}."
        need += [(b + "attn_norm.weight", GGML_F32, (H,)), (b + "ffn_norm.weight", GGML_F32, (H,))]
        need += [(b + m + ".weight", None, dims[m]) for m in LAYER_MATRICES]
    for name, gt, d in need:
        _check(g, name, gt, d)
    types = [P100_TYPE[g.tensors[n].ggml_type] for n in ("token_embd.weight", lm)]
    for l in range(cfg["n_layer"]):
        types += [P100_TYPE[g.tensors[f"blk.{l}.{m}.weight"].ggml_type] for m in LAYER_MATRICES]
    return lm, types


def load_llama(path, tp=None, max_ctx=None, kv_type=0, flags=0):
    """A Decoder holding the llama model of a GGUF file (this rank's slices
    under tensor parallelism).  Returns the decoder; the caller sets its
    state and closes it."""
    from . import Decoder, LlamaConfig, T_ATTN_NORM, T_EMBED, T_FFN_NORM, T_LM_HEAD, T_OUT_NORM, T_WDOWN, \
        T_WGATE_UP, T_WO, T_WQKV
    from .tp import k_shard, row_shard, split_range
    with GGUFFile(path) as g:
        kw, _ = llama_config(g, max_ctx, kv_type, flags)
        lm, types = llama_tensors(g, kw)
        uniform = all(t == types[0] for t in types)
        c = LlamaConfig(**kw, tensor_types=None if uniform else types)
        H, hd, F, V = c.hidden, c.head_dim, c.ffn, c.vocab
        nq, nkv = c.n_head, c.n_head_kv
        ntp = tp.size if tp is not None else 1
        rank = tp.rank if tp is not None else 0
        dec = Decoder(c, tp)
        try:
            def put(which, layer, data):
                ptr, nbytes, _, _ = dec.tensor(which, layer)
                data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
                if data.size != nbytes:
                    raise GGUFError(f"{path}: {data.size} bytes for a decoder tensor of {nbytes}")
                dec.write(ptr, data)

            def mat(name, dims):
                """(bytes, p100 format) of a matrix tensor, checked."""
                return _check(g, name, None, dims), P100_TYPE[g.tensors[name].ggml_type]

            put(T_EMBED, 0, _check(g, "token_embd.weight", None, (H, V)))
            put(T_OUT_NORM, 0, _check(g, "output_norm.weight", GGML_F32, (H,)))
            v0 = dec.vocab_offset
            vn = dec.tensor(T_LM_HEAD)[2]
            put(T_LM_HEAD, 0, row_shard(*mat(lm, (H, V)), V, H, v0, v0 + vn))
            q0, q1 = split_range(nq * hd, ntp, rank, hd)
            k0, k1 = split_range(nkv * hd, ntp, rank, hd)
            f0, f1 = split_range(F, ntp, rank, 256 if ntp > 1 else 1)
            for l in range(c.n_layer):
                b = f"blk.{l}."
                put(T_ATTN_NORM, l, _check(g, b + "attn_norm.weight", GGML_F32, (H,)))
                put(T_FFN_NORM, l, _check(g, b + "ffn_norm.weight", GGML_F32, (H,)))
                # fused matrices: each range in its own format, one after the other
                wq = row_shard(*mat(b + "attn_q.weight", (H, nq * hd)), nq * hd, H, q0, q1)
                wk = row_shard(*mat(b + "attn_k.weight", (H, nkv * hd)), nkv * hd, H, k0, k1)
                wv = row_shard(*mat(b + "attn_v.weight", (H, nkv * hd)), nkv * hd, H, k0, k1)
                put(T_WQKV, l, np.concatenate([wq, wk, wv]))
                put(T_WO, l, k_shard(*mat(b + "attn_output.weight", (nq * hd, H)), H, nq * hd, q0, q1))
                wg = row_shard(*mat(b + "ffn_gate.weight", (H, F)), F, H, f0, f1)
                wu = row_shard(*mat(b + "ffn_up.weight", (H, F)), F, H, f0, f1)
                put(T_WGATE_UP, l, np.concatenate([wg, wu]))
                put(T_WDOWN, l, k_shard(*mat(b + "ffn_down.weight", (F, H)), H, F, f0, f1))
        except BaseException:
            dec.close()
            raise
    return dec
