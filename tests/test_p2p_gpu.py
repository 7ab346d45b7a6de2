"""The peer-copy layer on B200 (reference: tests/test_p2p.cpp:69-210).

Single GPU: the Staged path of a same-device link (every chunk tail, stream
order, pinned-buffer reuse, destruction while work is queued).  Two GPUs: the
Peer path over NVLink both ways, and the forced Staged path
(P100_DISABLE_P2P=1); skipped with fewer devices.  Also the NCCL all-reduce of
the tensor-parallel layer across two ranks (one process per GPU)."""
import os
import socket

import numpy as np
import pytest

import p100_b200 as P

pytestmark = pytest.mark.gpu


def rand_bytes(torch, n, seed):
    return torch.from_numpy(np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)).cuda()


def test_probe_describes_every_device(cuda):
    text = P.p2p_describe()
    n = cuda.cuda.device_count()
    assert text.startswith(f"Devices: {n}")
    for i in range(n):
        assert cuda.cuda.get_device_name(i) in text


def test_staged_sizes_and_tails(cuda):
    maximum = 1 << 20
    src = rand_bytes(cuda, maximum, 7)
    dst = cuda.empty(maximum, dtype=cuda.uint8, device="cuda")
    stream = cuda.cuda.current_stream()
    link = P.PeerLink(0, 0, 4096)
    try:
        assert link.path == P.PATH_STAGED
        link.copy_async(dst.data_ptr(), src.data_ptr(), 0)
        for n in (0, 1, 4095, 4096, 4097, 14336, maximum):
            dst.fill_(0xD3)
            link.copy_async(dst.data_ptr(), src.data_ptr(), n, stream)
            got = dst.cpu()
            assert cuda.equal(got[:n], src[:n].cpu())
            assert bool((got[n:] == 0xD3).all())
    finally:
        link.close()


def test_stream_order_before(cuda):
    n = 1 << 20
    src = cuda.empty(n, dtype=cuda.uint8, device="cuda")
    dst = cuda.empty(n, dtype=cuda.uint8, device="cuda")
    link = P.PeerLink(0, 0, n)   # one chunk: the whole host-to-device copy is pending on return
    try:
        for _ in range(16):
            dst.zero_()
            src.fill_(0xAB)
            link.copy_async(dst.data_ptr(), src.data_ptr(), n)
            assert bool((dst.cpu() == 0xAB).all())
    finally:
        link.close()


def test_buffer_reuse_and_retiring_link(cuda):
    n, copies = 3 * 257 + 13, 64
    src = rand_bytes(cuda, n * copies, 29)
    dst = cuda.zeros(n * copies, dtype=cuda.uint8, device="cuda")
    link = P.PeerLink(0, 0, 257)
    try:
        for i in range(copies):
            link.copy_async(dst.data_ptr() + i * n, src.data_ptr() + i * n, n)
        assert cuda.equal(dst.cpu(), src.cpu())
    finally:
        link.close()
    # destruction waits for its own queued work without the caller synchronising
    dst.zero_()
    retiring = P.PeerLink(0, 0, 4096)
    retiring.copy_async(dst.data_ptr(), src.data_ptr(), n * copies)
    retiring.close()
    assert cuda.equal(dst.cpu(), src.cpu())


@pytest.mark.multigpu
def test_peer_both_ways_and_forced_staged(cuda, monkeypatch):
    if cuda.cuda.device_count() < 2:
        pytest.skip("peer path needs two GPUs")
    n = 3 * 4096 + 17
    for staged in (False, True):
        if staged:
            monkeypatch.setenv("P100_DISABLE_P2P", "1")
        else:
            monkeypatch.delenv("P100_DISABLE_P2P", raising=False)
        for s in (0, 1):
            d = 1 - s
            with cuda.cuda.device(s):
                src = rand_bytes(cuda, n, 41 + s)
            with cuda.cuda.device(d):
                dst = cuda.zeros(n, dtype=cuda.uint8, device=f"cuda:{d}")
            link = P.PeerLink(s, d, 4096)
            try:
                assert link.path == (P.PATH_STAGED if staged else P.PATH_PEER)
                with cuda.cuda.device(s):
                    link.copy_async(dst.data_ptr(), src.data_ptr(), n, cuda.cuda.current_stream(s))
                    cuda.cuda.synchronize(s)
            finally:
                link.close()
            cuda.cuda.synchronize(d)
            assert cuda.equal(dst.cpu(), src.cpu())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        box = [P.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = P.TP(box[0], world, rank, rank)
        x = torch.full((8192,), float(rank + 1), device=f"cuda:{rank}")
        tp.allreduce_sum(x)
        g = torch.empty(world * 4, device=f"cuda:{rank}")
        tp.allgather(torch.full((4,), float(rank), device=f"cuda:{rank}"), g)
        torch.cuda.synchronize()
        tp.close()
        q.put((rank, float(x[0]), float(x[-1]), g.cpu().tolist()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
def test_tp_allreduce_two_ranks(cuda):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert not p.is_alive()
    res = sorted(q.get() for _ in range(2))
    for rank, a, b, g in res:
        assert a == 3.0 and b == 3.0, res
        assert g == [0.0] * 4 + [1.0] * 4
