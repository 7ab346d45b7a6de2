"""p100_fa_decode_static: the FA decode for callers that may not allocate
device memory (their allocator owns the device budget, or they cannot afford
the synchronisation of cudaMalloc/cudaFree).  It keeps its split-K partials
in a fixed array inside the library instead of a caller workspace.

Both entry points run the same kernel with the same plan, so the outputs must
be the same bits as p100_fa_decode's (which takes a workspace): a difference
of any size would mean the partials, their (m, l) pairs or the merge tickets
sit at the wrong place in the array, or a previous call's leftovers leaked
in.  Each case runs twice in a row, and the cases run one after another, so
every call starts from what a call of another plan (another split, batch,
head size or cache format) left in the array.  One case is also held to the
attention tolerance of include/p100/tolerance.h against the CPU oracle's
attention_reference.

This file is collected last so a run stopped at its first failure has already
run everything else; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from conftest import ATTN_MAX_REL_TOL, lse_within_tolerance, out_within_tolerance

import oracle
import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu
STATIC_BYTES = 2 << 20   # P100_FA_STATIC_SCRATCH_BYTES


def static_decode():
    fn = P.lib().p100_fa_decode_static
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p] * 7 + [C.c_void_p]
    return fn


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


# (batch, n_head_q, n_head_kv, d, seq, cache capacity, kv_splits, kv_type); the
# plans: cluster merge (automatic split up to 8K keys), workspace merge
# (explicit splits), one part, the 8-warp shape past 8K keys, a q8_0 and a
# q4_0 cache of batch 2 with capacity > seq (explicit strides), d 64, and the
# SIMT kernel (d 256).
CASES = [
    (1, 32, 8, 128, 4096, 4096, 0, P.KV_F16),
    (1, 32, 8, 128, 1000, 1000, 7, P.KV_F16),
    (1, 32, 8, 128, 300, 300, 1, P.KV_F16),
    (1, 8, 2, 128, 12000, 12000, 0, P.KV_F16),
    (2, 16, 4, 128, 2999, 3001, 5, P.KV_Q8_0),
    (2, 16, 4, 64, 1500, 1537, 0, P.KV_Q4_0),
    (1, 64, 8, 64, 5000, 5000, 9, P.KV_F16),
    (2, 8, 4, 256, 700, 701, 3, P.KV_F16),
]


def inputs(cuda, batch, hq, hkv, d, seq, cap, kv_type, seed):
    q, k, v = W.attention_inputs(batch, hq, hkv, cap, d, seed=seed)
    if kv_type != P.KV_F16:
        k = W.kv_cache_blocks(kv_type, batch, hkv, cap, d, seed=seed + 1)
        v = W.kv_cache_blocks(kv_type, batch, hkv, cap, d, seed=seed + 2)
    return q, k, v, tuple(cuda.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b%d_h%d-%d_d%d_s%d_cap%d_sp%d_kv%d" % c)
def test_static_decode_bit_identical(cuda, case):
    batch, hq, hkv, d, seq, cap, splits, kv_type = case
    fn = static_decode()
    _, _, _, (qd, kd, vd) = inputs(cuda, batch, hq, hkv, d, seq, cap, kv_type, seed=seq + hq)
    desc = P.AttnDesc(batch=batch, n_head_q=hq, n_head_kv=hkv, seq_kv=seq, d_qk=d, d_v=d, kv_splits=splits,
                      kv_head_stride=cap * d, kv_batch_stride=hkv * cap * d, kv_type=kv_type)
    assert P.fa_workspace_size(desc) <= STATIC_BYTES   # the case fits the static array
    ref_o, ref_lse = P.fa_decode(desc, qd, kd, vd)
    ref_o, ref_lse = ref_o.cpu().numpy(), ref_lse.cpu().numpy()
    stream = C.c_void_p(cuda.cuda.current_stream().cuda_stream)
    for _ in range(2):   # the second call starts from the first call's leftovers
        o = cuda.full((batch, hq, 1, d), float("nan"), device="cuda")
        lse = cuda.full((batch, hq, 1), float("nan"), device="cuda")
        st = fn(C.byref(desc), ptr(qd), ptr(kd), ptr(vd), None, ptr(o), ptr(lse), stream)
        assert st == P.OK, P.last_error()
        assert np.array_equal(o.cpu().numpy().view(np.uint32), ref_o.view(np.uint32))
        assert np.array_equal(lse.cpu().numpy().view(np.uint32), ref_lse.view(np.uint32))
    assert P.device_error() == P.OK


def test_static_decode_against_attention_reference(cuda, orc):
    """GQA 4:1, d 128, 1000 keys over 7 parts (workspace merge) against the
    oracle's FP64 attention_reference, within tolerance.h."""
    fn = static_decode()
    q, k, v, (qd, kd, vd) = inputs(cuda, 1, 32, 8, 128, 1000, 1000, P.KV_F16, seed=5)
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=1000, kv_splits=7)
    stream = C.c_void_p(cuda.cuda.current_stream().cuda_stream)
    for _ in range(2):
        o = cuda.full((1, 32, 1, 128), float("nan"), device="cuda")
        lse = cuda.full((1, 32, 1), float("nan"), device="cuda")
        assert fn(C.byref(desc), ptr(qd), ptr(kd), ptr(vd), None, ptr(o), ptr(lse), stream) == P.OK, P.last_error()
        ref_o, ref_lse = orc.attention_reference(oracle.Attn(n_head_q=32, n_head_kv=8, seq_kv=1000), q,
                                                 k.astype(np.float32), v.astype(np.float32))
        got_o, got_lse = o.cpu().numpy().astype(np.float64), lse.cpu().numpy()
        assert out_within_tolerance(got_o, ref_o).all()
        assert lse_within_tolerance(got_lse, ref_lse).all()
        assert np.abs(got_o - ref_o).max() / np.abs(ref_o).max() <= ATTN_MAX_REL_TOL
    assert P.device_error() == P.OK


def test_static_decode_rejects_oversized_split(cuda):
    fn = static_decode()
    # 64 sequences x 8 kv heads x 64 parts x 4 heads x 128 floats > 2 MiB
    desc = P.AttnDesc(batch=64, n_head_q=32, n_head_kv=8, seq_kv=8192, kv_splits=64)
    need = P.fa_workspace_size(desc)
    assert need > STATIC_BYTES
    z = C.c_void_p(256)   # never dereferenced: the size check comes first
    st = fn(C.byref(desc), z, z, z, None, z, None, None)
    assert st == P.ERR_INVALID
    assert "static scratch" in P.last_error()
