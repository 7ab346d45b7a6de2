"""The reduce half of the one-shot peer all-reduce (p100_peer_reduce_rmsnorm),
on one GPU, through the C-ABI.

The graph decoder's tensor-parallel exchange stores every rank's partial sum
into every rank's slots as 64-bit words tagged with the exchange's epoch; the
next RMSNorm polls the tags, adds the ranks' values in rank order and
normalises.  Here the slots are an ordinary device buffer of one process,
filled by the test, so both outcomes of the bounded wait are tested without
a second GPU and without any fault: every word already tagged (the sum and
the bookkeeping), and words that never get their tag (a wait limit of a few
milliseconds: P100_ERR_TIMEOUT, and the next call is clean)."""
import ctypes as C

import numpy as np
import pytest

import p100_b200 as P

pytestmark = pytest.mark.gpu


def ptr(t):
    return C.c_void_p(t.data_ptr())


def tagged(values, epoch):
    """(epoch << 32) | fp32 bits, as int64 words."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((np.uint64(epoch) << np.uint64(32)) | bits).view(np.int64)


def reduce_call(cuda, x, w, k, xq, slots, world, rank, epoch, wait_ns):
    st = P.lib().p100_peer_reduce_rmsnorm(ptr(x), ptr(w), C.c_float(1e-5), k, ptr(xq), ptr(slots), world, rank,
                                          ptr(epoch), wait_ns, C.c_void_p(cuda.cuda.current_stream().cuda_stream))
    assert st == P.OK, P.last_error()


@pytest.mark.parametrize("k,world,rank", [(4096, 2, 0), (8192, 4, 3), (256, 8, 5)])
def test_reduce_sums_slots_in_rank_order(cuda, k, world, rank):
    rng = np.random.default_rng(k + world)
    x = rng.standard_normal(k).astype(np.float32)
    w = rng.uniform(0.9, 1.1, k).astype(np.float32)
    parts = (0.3 * rng.standard_normal((world, k))).astype(np.float32)
    # *epoch = 6: this exchange is e = 7 and reads slots [7 & 1]; the other
    # parity holds words of an older epoch that must not be read
    words = np.zeros((2, world, k), np.int64)
    words[1] = tagged(parts, 7)
    words[0] = tagged(rng.standard_normal((world, k)).astype(np.float32), 6)
    delta = parts[0].copy()
    for r in range(1, world):
        delta = (delta + parts[r]).astype(np.float32)
    xd, wd, sd = (cuda.from_numpy(a).cuda() for a in (x, w, words))
    xq = cuda.zeros(P.q8_1_bytes(k, 1), dtype=cuda.uint8, device="cuda")
    epoch = cuda.full((1,), 6, dtype=cuda.int32, device="cuda")
    assert P.device_error(clear=True) == P.OK
    reduce_call(cuda, xd, wd, k, xq, sd, world, rank, epoch, 0)
    # the same as x += delta (delta the rank-order sum) and the plain RMSNorm
    ref_x = cuda.from_numpy(x).cuda().view(1, k)
    ref_q = P.rmsnorm_q8_1(ref_x, wd, 1e-5, delta=cuda.from_numpy(delta).cuda().view(1, k))
    cuda.cuda.synchronize()
    assert np.array_equal(xd.cpu().numpy().view(np.uint32), ref_x.cpu().numpy().ravel().view(np.uint32))
    assert np.array_equal(xq.cpu().numpy(), ref_q.cpu().numpy().ravel())
    assert epoch.item() == 7
    assert P.device_error() == P.OK


def test_reduce_wait_runs_out_without_fault(cuda):
    """Two ranks' words that never get this exchange's tag: the wait gives up
    after its limit, the device flag reads P100_ERR_TIMEOUT, and the context
    stays usable (the next call, with its words tagged, is clean)."""
    k, world = 4096, 2
    x = cuda.ones(k, device="cuda")
    w = cuda.ones(k, device="cuda")
    slots = cuda.zeros(2 * world * k, dtype=cuda.int64, device="cuda")   # tag 0: nobody pushed
    xq = cuda.zeros(P.q8_1_bytes(k, 1), dtype=cuda.uint8, device="cuda")
    epoch = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert P.device_error(clear=True) == P.OK
    reduce_call(cuda, x, w, k, xq, slots, world, 0, epoch, 2_000_000)   # 2 ms
    assert P.device_error(clear=True) == P.ERR_TIMEOUT
    assert P.device_error() == P.OK
    epoch.fill_(0)
    words = np.zeros((2, world, k), np.int64)
    words[1] = tagged(np.full((world, k), 0.5, np.float32), 1)
    slots.copy_(cuda.from_numpy(words.ravel()))
    reduce_call(cuda, x, w, k, xq, slots, world, 0, epoch, 2_000_000)
    assert P.device_error() == P.OK
    assert epoch.item() == 1
    assert np.allclose(x.cpu().numpy(), 2.0)   # 1 + 0.5 + 0.5
