"""p100_fa_decode_static: the FA decode for callers that may not allocate
device memory (their allocator owns the device budget, or they cannot afford
the synchronisation of cudaMalloc/cudaFree).  It keeps its split-K partials
in a fixed array inside the library instead of a caller workspace.

Checked through the C-ABI against p100_fa_decode (which takes a workspace),
within the attention tolerance of include/p100/tolerance.h, on two calls in a
row — the second reuses the array with whatever the first left in it.  This
file is collected last so a run stopped at its first failure has already run
everything else; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from conftest import lse_within_tolerance, out_within_tolerance

import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu


def static_decode():
    fn = P.lib().p100_fa_decode_static
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p] * 7 + [C.c_void_p]
    return fn


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("seq,splits", [(4096, 0), (1000, 7), (300, 1)])
def test_static_decode_matches_workspace_decode(cuda, seq, splits):
    fn = static_decode()
    q, k, v = W.attention_inputs(1, 32, 8, seq, 128, seed=seq + 17)
    qd, kd, vd = (cuda.from_numpy(a).cuda() for a in (q, k, v))
    desc = P.AttnDesc(n_head_q=32, n_head_kv=8, seq_kv=seq, kv_splits=splits)
    ref_o, ref_lse = P.fa_decode(desc, qd, kd, vd)
    ref_o, ref_lse = ref_o.cpu().numpy(), ref_lse.cpu().numpy()
    stream = C.c_void_p(cuda.cuda.current_stream().cuda_stream)
    for _ in range(2):   # the second call starts from the first call's leftovers
        o = cuda.full((1, 32, 1, 128), float("nan"), device="cuda")
        lse = cuda.full((1, 32, 1), float("nan"), device="cuda")
        st = fn(C.byref(desc), ptr(qd), ptr(kd), ptr(vd), None, ptr(o), ptr(lse), stream)
        assert st == P.OK, P.last_error()
        got_o, got_lse = o.cpu().numpy(), lse.cpu().numpy()
        assert out_within_tolerance(got_o, ref_o.astype(np.float64)).all()
        assert lse_within_tolerance(got_lse, ref_lse).all()
    assert P.device_error() == P.OK


def test_static_decode_rejects_oversized_split(cuda):
    fn = static_decode()
    # 64 sequences x 8 kv heads x 64 parts x 4 heads x 128 floats > 2 MiB
    desc = P.AttnDesc(batch=64, n_head_q=32, n_head_kv=8, seq_kv=8192, kv_splits=64)
    need = P.fa_workspace_size(desc)
    assert need > (2 << 20)
    z = C.c_void_p(256)
    st = fn(C.byref(desc), z, z, z, None, z, None, None)
    assert st == P.ERR_INVALID
    assert "static scratch" in P.last_error()
