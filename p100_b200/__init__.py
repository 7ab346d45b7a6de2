"""p100_b200 — B200 (sm_100a) decode hot path of the P100 numerics contract.

The product is the C-ABI shared library ``p100_b200/lib/libp100_b200.so``
declared in ``include/p100/b200.h``.  This module is a thin ctypes view of it
for Python callers, tests and ``bench.py``: torch supplies device memory and
streams, every computation happens in the library's CUDA kernels, and there is
no CPU path — calls raise ``P100Error`` when the library or an sm_100 device
is missing.

Names follow the reference's contract (include/p100/qmv.h:17-49,
include/p100/attention.h:27-80): ``Q4_0/Q8_0/Q4_K`` block formats, Q8_1
activation blocks, ``AttnDesc`` mirroring ``AttnParams``.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import subprocess
import threading

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libp100_b200.so"
CSRC = HERE / "csrc"

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 4
TYPE_NAMES = {Q4_0: "q4_0", Q8_0: "q8_0", Q4_K: "q4_K", Q5_K: "q5_K", Q6_K: "q6_K"}
TYPES = {v: k for k, v in TYPE_NAMES.items()}
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}
# K/V cache element types (p100_kv_type) and their 32-value block bytes.
KV_F16, KV_Q8_0, KV_Q4_0 = 0, 1, 2
KV_BLOCK_BYTES = {KV_Q8_0: 34, KV_Q4_0: 18}
Q8_1_BLOCK_BYTES = 36
QMV_PDL = 1
QMV_TC = 2   # P100_QMV_TC: batch 2..16 on the tcgen05 kernel wherever it fits
QMV_MMA = 4  # P100_QMV_MMA: batch 2..16 never on the tcgen05 kernel
TP_PEER_MAX = 65536   # P100_TP_PEER_MAX: all-reduces up to this count may run over peer memory

STATUS = {0: "P100_OK", 1: "P100_ERR_INVALID", 2: "P100_ERR_CUDA", 3: "P100_ERR_NCCL",
          4: "P100_ERR_TIMEOUT", 5: "P100_ERR_UNSUPPORTED"}
OK, ERR_INVALID, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_UNSUPPORTED = range(6)
PATH_PEER, PATH_STAGED = 0, 1
TP_ID_BYTES = 128


class P100Error(RuntimeError):
    """A non-OK p100_status, with p100_last_error()'s text."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


class InvalidArgument(P100Error, ValueError):
    """P100_ERR_INVALID — the reference raises std::invalid_argument here."""


class AttnDesc(C.Structure):
    """p100_attn_desc: AttnParams (include/p100/attention.h:27-41) + split/strides."""
    _fields_ = [("batch", C.c_int), ("n_head_q", C.c_int), ("n_head_kv", C.c_int), ("seq_q", C.c_int),
                ("seq_kv", C.c_int), ("d_qk", C.c_int), ("d_v", C.c_int), ("scale", C.c_float),
                ("softcap", C.c_float), ("causal", C.c_int), ("kv_splits", C.c_int),
                ("kv_head_stride", C.c_longlong), ("kv_batch_stride", C.c_longlong), ("kv_type", C.c_int)]

    def __init__(self, batch=1, n_head_q=1, n_head_kv=1, seq_q=1, seq_kv=1, d_qk=128, d_v=128, scale=0.0,
                 softcap=0.0, causal=False, kv_splits=0, kv_head_stride=0, kv_batch_stride=0, kv_type=0):
        super().__init__(batch, n_head_q, n_head_kv, seq_q, seq_kv, d_qk, d_v, scale, softcap, int(bool(causal)),
                         kv_splits, kv_head_stride, kv_batch_stride, kv_type)


_lib = None
_lock = threading.Lock()


def build(verbose=False):
    """Compile the CUDA library for sm_100a (nvcc cross-compiles without a GPU)."""
    out = None if verbose else subprocess.DEVNULL
    subprocess.run(["make", "-s", "-C", str(CSRC)], check=True, stdout=out)


def _bind(lib):
    vp, ip, sz, st = C.c_void_p, C.c_int, C.c_size_t, C.c_void_p
    sigs = {
        "p100_abi_version": (ip, []),
        "p100_last_error": (C.c_char_p, []),
        "p100_status_name": (C.c_char_p, [ip]),
        "p100_device_check": (ip, [ip]),
        "p100_device_error": (ip, [ip]),
        "p100_block_elems": (ip, [ip]),
        "p100_block_bytes": (ip, [ip]),
        "p100_weight_bytes": (sz, [ip, ip, ip]),
        "p100_q8_1_bytes": (sz, [ip, ip]),
        "p100_q8_1_quantize": (ip, [vp, vp, ip, ip, st]),
        "p100_dequantize": (ip, [ip, vp, ip, ip, vp, st]),
        "p100_qmv": (ip, [ip, vp, ip, ip, vp, ip, vp, st]),
        "p100_qmv_ex": (ip, [ip, vp, ip, ip, vp, ip, vp, C.c_uint, st]),
        "p100_qmv_f32": (ip, [ip, vp, ip, ip, vp, ip, vp, vp, C.c_uint, st]),
        "p100_q8_1_quantize_ex": (ip, [vp, vp, ip, ip, C.c_uint, st]),
        "p100_h16_prepare": (ip, [vp, vp, vp, ip, ip, st]),
        "p100_qmv_h16": (ip, [ip, vp, ip, ip, vp, vp, ip, ip, vp, st]),
        "p100_attn_validate": (ip, [vp, C.c_char_p, sz]),
        "p100_fa_workspace_size": (sz, [vp]),
        "p100_fa_workspace_init": (ip, [vp, sz, st]),
        "p100_fa_decode": (ip, [vp, vp, vp, vp, vp, vp, vp, vp, sz, st]),
        "p100_kv_to_f16": (ip, [ip, vp] + [C.c_longlong] * 7 + [vp, st]),
        "p100_tp_unique_id": (ip, [vp]),
        "p100_tp_init_rank": (ip, [vp, ip, ip, ip, C.POINTER(vp)]),
        "p100_tp_create": (ip, [ip, C.POINTER(ip), C.POINTER(vp)]),
        "p100_tp_rank": (ip, [vp]),
        "p100_tp_size": (ip, [vp]),
        "p100_tp_device": (ip, [vp]),
        "p100_tp_peer": (ip, [vp]),
        "p100_tp_allreduce_sum": (ip, [vp, vp, sz, st]),
        "p100_tp_allreduce_sum_group": (ip, [C.POINTER(vp), ip, C.POINTER(vp), sz, C.POINTER(vp)]),
        "p100_tp_allgather": (ip, [vp, vp, vp, sz, st]),
        "p100_tp_destroy": (ip, [vp]),
        "p100_p2p_describe": (sz, [C.c_char_p, sz]),
        "p100_p2p_disabled_by_env": (ip, []),
        "p100_peer_link_create": (ip, [ip, ip, sz, C.POINTER(vp)]),
        "p100_peer_link_path": (ip, [vp]),
        "p100_peer_link_copy": (ip, [vp, vp, vp, sz, st]),
        "p100_peer_link_destroy": (ip, [vp]),
        "p100_rmsnorm_q8_1": (ip, [vp, vp, vp, C.c_float, ip, ip, vp, vp, st]),
        "p100_peer_reduce_rmsnorm": (ip, [vp, vp, C.c_float, ip, vp, vp, ip, ip, vp, C.c_ulonglong, st]),
        "p100_qmv_rmsnorm": (ip, [ip, vp, ip, ip, vp, vp, vp, vp, C.c_float, vp, C.c_uint, st]),
        "p100_rope_table": (None, [vp, ip, ip, C.c_float]),
        "p100_rope_kv_append": (ip, [vp, ip, ip, ip, vp, ip, vp, vp, vp, C.c_longlong, st]),
        "p100_swiglu_q8_1": (ip, [vp, ip, ip, vp, st]),
        "p100_argmax": (ip, [vp, ip, ip, vp, vp, st]),
        "p100_decoder_create": (ip, [vp, vp, C.POINTER(vp)]),
        "p100_decoder_init_random": (ip, [vp, C.c_ulonglong]),
        "p100_decoder_fill_kv": (ip, [vp, ip, C.c_ulonglong, C.c_float]),
        "p100_decoder_set_state": (ip, [vp, ip, ip]),
        "p100_decoder_state": (ip, [vp, C.POINTER(ip), C.POINTER(ip)]),
        "p100_decoder_step": (ip, [vp, ip, st]),
        "p100_decoder_tensor": (ip, [vp, ip, ip, C.POINTER(vp), C.POINTER(sz), C.POINTER(ip), C.POINTER(ip)]),
        "p100_decoder_buffer": (ip, [vp, ip, C.POINTER(vp), C.POINTER(sz)]),
        "p100_decoder_vocab_offset": (ip, [vp]),
        "p100_decoder_path": (ip, [vp]),
        "p100_decoder_weight_bytes_per_token": (sz, [vp]),
        "p100_decoder_destroy": (ip, [vp]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib():
    """The loaded C-ABI library.  Raises P100Error when it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise P100Error(ERR_UNSUPPORTED, f"{LIB_PATH} is not built (python -c 'import p100_b200; "
                                                     "p100_b200.build()')")
                _lib = _bind(C.CDLL(str(LIB_PATH)))
    return _lib


def symbols():
    """Every symbol include/p100/b200.h declares, in header order."""
    import re
    text = (HERE.parent / "include" / "p100" / "b200.h").read_text()
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\**(p100_[a-z0-9_]+)\(", text, re.M)


def last_error():
    return lib().p100_last_error().decode()


def check(status):
    if status != OK:
        cls = InvalidArgument if status == ERR_INVALID else P100Error
        raise cls(status, last_error())
    return status


# ---------------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def device_check(device=0):
    return lib().p100_device_check(device)


def device_error(clear=True):
    """P100_ERR_TIMEOUT if a kernel gave up a bounded wait (synchronises)."""
    return lib().p100_device_error(int(clear))


def weight_bytes(qtype, rows, k):
    return lib().p100_weight_bytes(qtype, rows, k)


def q8_1_bytes(k, batch=1):
    return lib().p100_q8_1_bytes(k, batch)


def q8_1_quantize(x, out=None, stream=None, flags=0):
    """Q8_1 blocks of x (fp32 [batch, k] on the GPU) -> uint8 [batch * k/32 * 36]
    (p100_q8_1_quantize, or p100_q8_1_quantize_ex with flags)."""
    torch = _torch()
    x = x.contiguous()
    k = x.shape[-1]
    batch = x.numel() // k
    if out is None:
        out = torch.empty(batch * (k // 32) * Q8_1_BLOCK_BYTES, dtype=torch.uint8, device=x.device)
    if flags:
        check(lib().p100_q8_1_quantize_ex(_ptr(x), _ptr(out), k, batch, flags, _stream(stream)))
    else:
        check(lib().p100_q8_1_quantize(_ptr(x), _ptr(out), k, batch, _stream(stream)))
    return out


def h16_prepare(x, stream=None):
    """h16 activations of x (fp32 [batch, k] on the GPU): (h fp16 [batch, k] in
    the stored 0,2,1,3 order, ss fp32 [batch, k/32, 2] {scale, sum})
    (p100_h16_prepare, qmv::prepare's h16 fields)."""
    torch = _torch()
    x = x.contiguous()
    k = x.shape[-1]
    batch = x.numel() // k
    h = torch.empty(batch, k, dtype=torch.float16, device=x.device)
    ss = torch.empty(batch, k // 32, 2, dtype=torch.float32, device=x.device)
    check(lib().p100_h16_prepare(_ptr(x), _ptr(h), _ptr(ss), k, batch, _stream(stream)))
    return h, ss


def qmv_h16(qtype, w, rows, k, h, ss, batch=1, chain=16, y=None, stream=None):
    """y[batch, rows] = qmv::h16_model with HFMA2 chains of `chain` (p100_qmv_h16)."""
    torch = _torch()
    if y is None:
        y = torch.empty(batch, rows, dtype=torch.float32, device=h.device)
    check(lib().p100_qmv_h16(qtype, _ptr(w), rows, k, _ptr(h), _ptr(ss), batch, chain, _ptr(y), _stream(stream)))
    return y


def dequantize(qtype, w, rows, k, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty(rows, k, dtype=torch.float32, device=w.device)
    check(lib().p100_dequantize(qtype, _ptr(w), rows, k, _ptr(out), _stream(stream)))
    return out


def qmv(qtype, w, rows, k, x_q8_1, batch=1, y=None, flags=0, stream=None):
    """y[batch, rows] = W x for Q8_1 activations (p100_qmv / p100_qmv_ex)."""
    torch = _torch()
    if y is None:
        y = torch.empty(batch, rows, dtype=torch.float32, device=w.device)
    check(lib().p100_qmv_ex(qtype, _ptr(w), rows, k, _ptr(x_q8_1), batch, _ptr(y), flags, _stream(stream)))
    return y


def qmv_f32(qtype, w, rows, k, x, batch=1, y=None, x_q8_1=None, flags=0, stream=None):
    """y[batch, rows] = W . Q8_1(x) for fp32 x (p100_qmv_f32): with x_q8_1,
    the quantiser into it and the mat-vec as its programmatic dependent;
    without, one fused launch (batch 1 on the team kernel only)."""
    torch = _torch()
    if y is None:
        y = torch.empty(batch, rows, dtype=torch.float32, device=w.device)
    check(lib().p100_qmv_f32(qtype, _ptr(w), rows, k, _ptr(x), batch, _ptr(x_q8_1), _ptr(y), flags,
                             _stream(stream)))
    return y


def attn_validate(desc):
    buf = C.create_string_buffer(256)
    st = lib().p100_attn_validate(C.byref(desc), buf, 256)
    return st == OK, buf.value.decode()


def fa_workspace_size(desc):
    return lib().p100_fa_workspace_size(C.byref(desc))


def fa_workspace(desc, device=None, stream=None):
    """A zero-initialised workspace for desc (None if none is needed)."""
    torch = _torch()
    n = fa_workspace_size(desc)
    if n == 0:
        return None   # none needed, or an invalid desc that p100_fa_decode reports with its status
    return torch.zeros(n, dtype=torch.uint8, device=device or "cuda")


def kv_to_f16(kv_type, src, ne00, ne01, ne02=1, ne03=1, s01=None, s02=None, s03=None, out=None, stream=None):
    """Quantised K/V view (uint8 blocks) -> fp16 [ne03, ne02, ne01, ne00] (p100_kv_to_f16);
    block strides default to a contiguous view."""
    torch = _torch()
    nb = ne00 // 32
    s01 = nb if s01 is None else s01
    s02 = nb * ne01 if s02 is None else s02
    s03 = s02 * ne02 if s03 is None else s03
    if out is None:
        out = torch.empty(ne03, ne02, ne01, ne00, dtype=torch.float16, device=src.device)
    check(lib().p100_kv_to_f16(kv_type, _ptr(src), ne00, ne01, ne02, ne03, s01, s02, s03, _ptr(out),
                               _stream(stream)))
    return out


def fa_decode(desc, q, k, v, mask=None, o=None, lse=None, ws=None, stream=None):
    """Split-K FA-vec decode: q fp32 [B,Hq,1,D], k/v fp16 [B,Hkv,S,D] (or, with desc.kv_type
    KV_Q8_0 / KV_Q4_0, uint8 blocks of the same rows) -> o fp32, lse fp32."""
    torch = _torch()
    if o is None:
        o = torch.empty(desc.batch, desc.n_head_q, desc.seq_q, desc.d_v, dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty(desc.batch, desc.n_head_q, desc.seq_q, dtype=torch.float32, device=q.device)
    if ws is None:
        ws = fa_workspace(desc, q.device)
    nbytes = ws.numel() if ws is not None else 0
    check(lib().p100_fa_decode(C.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(mask), _ptr(o), _ptr(lse),
                               _ptr(ws), nbytes, _stream(stream)))
    return o, lse


# ---------------------------------------------------------------- tensor parallel
def tp_unique_id():
    buf = (C.c_ubyte * TP_ID_BYTES)()
    check(lib().p100_tp_unique_id(buf))
    return bytes(buf)


class TP:
    """One rank of a row-split tensor-parallel group (p100_tp_*)."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        h = C.c_void_p()
        buf = (C.c_ubyte * TP_ID_BYTES).from_buffer_copy(uid)
        check(lib().p100_tp_init_rank(buf, nranks, rank, device, C.byref(h)))
        self.handle = h

    @property
    def rank(self):
        return lib().p100_tp_rank(self.handle)

    @property
    def size(self):
        return lib().p100_tp_size(self.handle)

    @property
    def peer(self):
        """True when all-reduces of up to TP_PEER_MAX values run over peer memory."""
        return bool(lib().p100_tp_peer(self.handle))

    def allreduce_sum(self, buf, stream=None):
        check(lib().p100_tp_allreduce_sum(self.handle, _ptr(buf), buf.numel(), _stream(stream)))
        return buf

    def allgather(self, inp, out, stream=None):
        check(lib().p100_tp_allgather(self.handle, _ptr(inp), _ptr(out), inp.numel(), _stream(stream)))
        return out

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            check(lib().p100_tp_destroy(h))


# ------------------------------------------------------------ decode-step glue
def rmsnorm_q8_1(x, w, eps, delta=None, y_out=None, xq=None, stream=None):
    """x += delta (in place, when given); Q8_1 of RMSNorm(x) * w (p100_rmsnorm_q8_1)."""
    torch = _torch()
    k = x.shape[-1]
    batch = x.numel() // k
    if xq is None:
        xq = torch.empty(batch * (k // 32) * Q8_1_BLOCK_BYTES, dtype=torch.uint8, device=x.device)
    check(lib().p100_rmsnorm_q8_1(_ptr(x), _ptr(delta), _ptr(w), eps, k, batch, _ptr(xq), _ptr(y_out),
                                  _stream(stream)))
    return xq


def qmv_rmsnorm(qtype, w, rows, k, x_in, norm_w, eps, delta=None, x_out=None, y=None, flags=0, stream=None):
    """y = W * Q8_1(RMSNorm(x_in + delta) * norm_w), x_in + delta into x_out
    (p100_qmv_rmsnorm: the RMSNorm fused into the batch-1 mat-vec)."""
    torch = _torch()
    if y is None:
        y = torch.empty(1, rows, dtype=torch.float32, device=x_in.device)
    check(lib().p100_qmv_rmsnorm(qtype, _ptr(w), rows, k, _ptr(x_in), _ptr(delta), _ptr(x_out), _ptr(norm_w), eps,
                                 _ptr(y), flags, _stream(stream)))
    return y


def rope_table(max_pos, head_dim, theta):
    """Host numpy [max_pos, head_dim/2, 2] (cos, sin) table (p100_rope_table)."""
    import numpy as np
    out = np.zeros((max_pos, head_dim // 2, 2), dtype=np.float32)
    lib().p100_rope_table(out.ctypes.data_as(C.c_void_p), max_pos, head_dim, theta)
    return out


def rope_kv_append(qkv, n_head, n_head_kv, head_dim, rope_cs, max_pos, pos_dev, k_cache, v_cache,
                   kv_head_stride, stream=None):
    check(lib().p100_rope_kv_append(_ptr(qkv), n_head, n_head_kv, head_dim, _ptr(rope_cs), max_pos, _ptr(pos_dev),
                                    _ptr(k_cache), _ptr(v_cache), kv_head_stride, _stream(stream)))


def swiglu_q8_1(gate_up, n, xq=None, stream=None):
    torch = _torch()
    batch = gate_up.numel() // (2 * n)
    if xq is None:
        xq = torch.empty(batch * (n // 32) * Q8_1_BLOCK_BYTES, dtype=torch.uint8, device=gate_up.device)
    check(lib().p100_swiglu_q8_1(_ptr(gate_up), n, batch, _ptr(xq), _stream(stream)))
    return xq


def argmax(x, stream=None):
    """(idx int32 [batch], val fp32 [batch]) of the rows of x (p100_argmax)."""
    torch = _torch()
    n = x.shape[-1]
    batch = x.numel() // n
    idx = torch.empty(batch, dtype=torch.int32, device=x.device)
    val = torch.empty(batch, dtype=torch.float32, device=x.device)
    check(lib().p100_argmax(_ptr(x), n, batch, _ptr(idx), _ptr(val), _stream(stream)))
    return idx, val


class LlamaConfig(C.Structure):
    """p100_llama_config."""
    _fields_ = [("n_layer", C.c_int), ("hidden", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("max_ctx", C.c_int),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("wtype", C.c_int), ("flags", C.c_int),
                ("kv_type", C.c_int), ("tensor_types", C.POINTER(C.c_int))]

    def __init__(self, n_layer, hidden, n_head, n_head_kv, head_dim, ffn, vocab, max_ctx, rope_theta=500000.0,
                 norm_eps=1e-5, wtype=0, flags=0, kv_type=0, tensor_types=None):
        """tensor_types: None (wtype everywhere) or DEC_TENSOR_TYPES(n_layer)
        formats indexed by TT_EMBED, TT_LM_HEAD and tt_layer(l, TT_Q ..)."""
        super().__init__(n_layer, hidden, n_head, n_head_kv, head_dim, ffn, vocab, max_ctx, rope_theta, norm_eps,
                         wtype, flags, kv_type)
        self.set_tensor_types(tensor_types)

    def set_tensor_types(self, types):
        if types is None:
            self._tt = None
            self.tensor_types = None
            return
        types = [int(t) for t in types]
        if len(types) != dec_tensor_types(self.n_layer):
            raise ValueError(f"tensor_types needs {dec_tensor_types(self.n_layer)} entries, got {len(types)}")
        self._tt = (C.c_int * len(types))(*types)   # kept alive with the config
        self.tensor_types = C.cast(self._tt, C.POINTER(C.c_int))

    def types(self):
        """The format of every tensor id (wtype where tensor_types is None)."""
        if self._tt is None:
            return [self.wtype] * dec_tensor_types(self.n_layer)
        return list(self._tt)


DEC_FUSED_NORM = 1   # P100_DEC_FUSED_NORM
DEC_STEP = 2         # P100_DEC_STEP: the persistent step kernel where it applies (opt-in)
DEC_PATH_GRAPH, DEC_PATH_STEP = 0, 1   # p100_decoder_path
# tensor ids of LlamaConfig.tensor_types (P100_TT_*)
TT_EMBED, TT_LM_HEAD = 0, 1
TT_Q, TT_K, TT_V, TT_O, TT_GATE, TT_UP, TT_DOWN = range(7)


def tt_layer(layer, part):
    return 2 + 7 * layer + part


def dec_tensor_types(n_layer):
    return 2 + 7 * n_layer


T_EMBED, T_ATTN_NORM, T_WQKV, T_WO, T_FFN_NORM, T_WGATE_UP, T_WDOWN, T_OUT_NORM, T_LM_HEAD = range(9)
B_HIDDEN, B_LOGITS, B_KCACHE, B_VCACHE, B_ROPE = range(5)


class Decoder:
    """A batch-1 Llama-shaped decoder (p100_decoder_*), one GPU or one TP rank."""

    def __init__(self, cfg: LlamaConfig, tp: "TP | None" = None):
        h = C.c_void_p()
        self.cfg = cfg
        check(lib().p100_decoder_create(C.byref(cfg), tp.handle if tp is not None else None, C.byref(h)))
        self.handle = h

    def init_random(self, seed):
        check(lib().p100_decoder_init_random(self.handle, seed))

    def fill_kv(self, n_pos, seed, scale=0.5):
        check(lib().p100_decoder_fill_kv(self.handle, n_pos, seed, scale))

    def set_state(self, pos, token):
        check(lib().p100_decoder_set_state(self.handle, pos, token))

    def state(self):
        pos, tok = C.c_int(), C.c_int()
        check(lib().p100_decoder_state(self.handle, C.byref(pos), C.byref(tok)))
        return pos.value, tok.value

    def step(self, n=1, stream=None):
        check(lib().p100_decoder_step(self.handle, n, _stream(stream)))

    def tensor(self, which, layer=0):
        """(device address, bytes, rows, cols) of a weight tensor."""
        ptr, n, rows, cols = C.c_void_p(), C.c_size_t(), C.c_int(), C.c_int()
        check(lib().p100_decoder_tensor(self.handle, layer, which, C.byref(ptr), C.byref(n), C.byref(rows),
                                        C.byref(cols)))
        return ptr.value, n.value, rows.value, cols.value

    def buffer(self, which):
        ptr, n = C.c_void_p(), C.c_size_t()
        check(lib().p100_decoder_buffer(self.handle, which, C.byref(ptr), C.byref(n)))
        return ptr.value, n.value

    @property
    def path(self):
        """DEC_PATH_STEP (one persistent kernel a token) or DEC_PATH_GRAPH."""
        return lib().p100_decoder_path(self.handle)

    @property
    def vocab_offset(self):
        return lib().p100_decoder_vocab_offset(self.handle)

    @property
    def weight_bytes_per_token(self):
        return lib().p100_decoder_weight_bytes_per_token(self.handle)

    def read(self, ptr, nbytes):
        """Host bytes (numpy uint8) of nbytes at a device address (synchronises)."""
        return device_to_host(ptr, nbytes)

    def write(self, ptr, data):
        """Copy host bytes (numpy array) to a device address (synchronises)."""
        host_to_device(ptr, data)

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            check(lib().p100_decoder_destroy(h))


def _runtime():
    from cuda.bindings import runtime as rt   # cuda-python: raw-address copies for tests and tools
    return rt


def device_to_host(ptr, nbytes):
    """numpy uint8 copy of nbytes at a device address (cudaMemcpy, synchronous)."""
    import numpy as np
    rt = _runtime()
    out = np.empty(nbytes, dtype=np.uint8)
    (err,) = rt.cudaMemcpy(out.ctypes.data, ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    if int(err) != 0:
        raise P100Error(ERR_CUDA, f"cudaMemcpy device to host failed ({err})")
    return out


def host_to_device(ptr, data):
    import numpy as np
    rt = _runtime()
    data = np.ascontiguousarray(data)
    (err,) = rt.cudaMemcpy(ptr, data.ctypes.data, data.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    if int(err) != 0:
        raise P100Error(ERR_CUDA, f"cudaMemcpy host to device failed ({err})")


# ---------------------------------------------------------------- peer copies
def p2p_describe():
    n = lib().p100_p2p_describe(None, 0)
    if n == 0:
        raise P100Error(ERR_CUDA, last_error())
    buf = C.create_string_buffer(n)
    lib().p100_p2p_describe(buf, n)
    return buf.value.decode()


class PeerLink:
    """p100::p2p::PeerLink (include/p100/p2p.h) through the C view."""

    def __init__(self, src_dev, dst_dev, chunk_bytes=4 << 20):
        h = C.c_void_p()
        check(lib().p100_peer_link_create(src_dev, dst_dev, chunk_bytes, C.byref(h)))
        self.handle = h

    @property
    def path(self):
        return lib().p100_peer_link_path(self.handle)

    def copy_async(self, dst_ptr, src_ptr, nbytes, stream=None):
        check(lib().p100_peer_link_copy(self.handle, C.c_void_p(dst_ptr), C.c_void_p(src_ptr), nbytes,
                                        _stream(stream)))

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            check(lib().p100_peer_link_destroy(h))
