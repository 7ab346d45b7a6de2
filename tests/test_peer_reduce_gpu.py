"""The reduce half of the one-shot peer all-reduce (p100_peer_reduce_rmsnorm),
on one GPU, through the C-ABI.

The graph decoder's tensor-parallel exchange stores every rank's partial sum
into every rank's slots and counts the arrivals on each rank's counter; the
next RMSNorm waits for the count, adds the slots in rank order and
normalises.  Here the slots and the counter are ordinary device buffers of
one process, so both outcomes of the bounded wait are tested without a
second GPU and without any fault: arrivals already counted (the sum and the
bookkeeping), and arrivals that never come (a counter nobody raises, a wait
limit of a few milliseconds: P100_ERR_TIMEOUT, and the next call is clean)."""
import ctypes as C

import numpy as np
import pytest

import p100_b200 as P

pytestmark = pytest.mark.gpu


def ptr(t):
    return C.c_void_p(t.data_ptr())


def reduce_call(cuda, x, w, k, xq, slots, world, rank, epoch, count, done, arrivals, wait_ns):
    st = P.lib().p100_peer_reduce_rmsnorm(ptr(x), ptr(w), C.c_float(1e-5), k, ptr(xq), ptr(slots), world, rank,
                                          ptr(epoch), ptr(count), ptr(done), arrivals, wait_ns,
                                          C.c_void_p(cuda.cuda.current_stream().cuda_stream))
    assert st == P.OK, P.last_error()


@pytest.mark.parametrize("k,world,rank", [(4096, 2, 0), (8192, 4, 3), (256, 8, 5)])
def test_reduce_sums_slots_in_rank_order(cuda, k, world, rank):
    rng = np.random.default_rng(k + world)
    x = rng.standard_normal(k).astype(np.float32)
    w = rng.uniform(0.9, 1.1, k).astype(np.float32)
    slots = (0.3 * rng.standard_normal((2, world, k))).astype(np.float32)
    par = 1   # *epoch = 0, so this exchange is e = 1 and reads slots[1]
    delta = slots[par, 0].copy()
    for r in range(1, world):
        delta = (delta + slots[par, r]).astype(np.float32)
    xd, wd, sd = (cuda.from_numpy(a).cuda() for a in (x, w, slots))
    xq = cuda.zeros(P.q8_1_bytes(k, 1), dtype=cuda.uint8, device="cuda")
    epoch = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    count = cuda.full((1,), 5 * world, dtype=cuda.int64, device="cuda")   # every arrival already counted
    done = cuda.full((1,), 4 * world, dtype=cuda.int64, device="cuda")
    assert P.device_error(clear=True) == P.OK
    reduce_call(cuda, xd, wd, k, xq, sd, world, rank, epoch, count, done, world, 0)
    # the same as x += delta (delta the rank-order sum) and the plain RMSNorm
    ref_x = cuda.from_numpy(x).cuda().view(1, k)
    ref_q = P.rmsnorm_q8_1(ref_x, wd, 1e-5, delta=cuda.from_numpy(delta).cuda().view(1, k))
    cuda.cuda.synchronize()
    assert np.array_equal(xd.cpu().numpy().view(np.uint32), ref_x.cpu().numpy().ravel().view(np.uint32))
    assert np.array_equal(xq.cpu().numpy(), ref_q.cpu().numpy().ravel())
    assert epoch.item() == 1 and done.item() == 5 * world and count.item() == 5 * world
    assert P.device_error() == P.OK


def test_reduce_wait_runs_out_without_fault(cuda):
    """Two ranks' arrivals that never come: the wait gives up after its
    limit, the device flag reads P100_ERR_TIMEOUT, and the context stays
    usable (the next call, with its arrivals counted, is clean)."""
    k, world = 4096, 2
    x = cuda.ones(k, device="cuda")
    w = cuda.ones(k, device="cuda")
    slots = cuda.zeros(2 * world * k, device="cuda")
    xq = cuda.zeros(P.q8_1_bytes(k, 1), dtype=cuda.uint8, device="cuda")
    epoch = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    count = cuda.zeros(1, dtype=cuda.int64, device="cuda")   # nobody ever arrives
    done = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    assert P.device_error(clear=True) == P.OK
    reduce_call(cuda, x, w, k, xq, slots, world, 0, epoch, count, done, world, 2_000_000)   # 2 ms
    assert P.device_error(clear=True) == P.ERR_TIMEOUT
    assert P.device_error() == P.OK
    count.fill_(10 * world)
    done.fill_(0)
    reduce_call(cuda, x, w, k, xq, slots, world, 0, epoch, count, done, world, 2_000_000)
    assert P.device_error() == P.OK
    assert done.item() == world
