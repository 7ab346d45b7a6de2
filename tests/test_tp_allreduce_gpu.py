"""p100_tp_allreduce_sum over NVLink peer memory, one process per GPU.

A group joined with p100_tp_init_rank whose GPUs all reach each other runs
all-reduces of up to P100_TP_PEER_MAX values as one kernel: every rank's
values go to every rank as epoch-tagged 64-bit words, and each rank adds
them in rank order.  So the result is the float32 sum x_0 + x_1 + ... in
that order, bit for bit, on every rank.  Checked here on three calls in a
row (the epoch advances, the slots alternate), inside a CUDA graph replayed
twice, at ragged counts (1, 7, 8191) and at the limit; counts past the limit
and P100_TP_ALLREDUCE=nccl take ncclAllReduce (its summation order is its
own: within 1e-6 relative)."""
import os
import socket

import numpy as np
import pytest

import p100_b200 as P

pytestmark = pytest.mark.gpu

COUNTS = [1, 7, 4096, 8191, 16384, P.TP_PEER_MAX, P.TP_PEER_MAX + 1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(count, rank, call):
    rng = np.random.default_rng(1_000_003 * count + 101 * rank + call)
    return rng.standard_normal(count).astype(np.float32)


def _rank_order_sum(count, world, call):
    s = _inputs(count, 0, call)
    for r in range(1, world):
        s = (s + _inputs(count, r, call)).astype(np.float32)
    return s


def _rank(rank, world, port, q, mode):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", P100_TP_ALLREDUCE=mode)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    tp = None
    try:
        box = [P.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = P.TP(box[0], world, rank, rank)
        out = {"peer": tp.peer, "eager": {}, "graph": []}
        for count in COUNTS:
            got = []
            for call in range(3):
                x = torch.from_numpy(_inputs(count, rank, call)).cuda()
                tp.allreduce_sum(x)
                got.append(x.cpu().numpy())
            out["eager"][count] = got
        # two all-reduces captured in one graph, replayed with new inputs
        a = torch.empty(8191, device="cuda")
        b = torch.empty(16384, device="cuda")
        a.copy_(torch.from_numpy(_inputs(8191, rank, 10)))
        b.copy_(torch.from_numpy(_inputs(16384, rank, 10)))
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            tp.allreduce_sum(a)
            tp.allreduce_sum(b)
        for call in (11, 12):
            a.copy_(torch.from_numpy(_inputs(8191, rank, call)))
            b.copy_(torch.from_numpy(_inputs(16384, rank, call)))
            g.replay()
            torch.cuda.synchronize()
            out["graph"].append((call, a.cpu().numpy(), b.cpu().numpy()))
        del g   # the graph goes before the communicator
        torch.cuda.synchronize()
        out["device_error"] = P.device_error()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


def _run(cuda, world, mode):
    if cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    for rank, out in res:
        assert isinstance(out, dict), (rank, out)
    return [out for _, out in res]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_rank_order_bits(cuda, world):
    outs = _run(cuda, world, "peer")
    for out in outs:
        assert out["peer"]
        assert out["device_error"] == P.OK
        for count in COUNTS:
            for call in range(3):
                want = _rank_order_sum(count, world, call)
                got = out["eager"][count][call]
                if count <= P.TP_PEER_MAX:
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (count, call)
                else:   # NCCL
                    assert np.allclose(got, want, rtol=1e-6, atol=1e-6 * world), (count, call)
        for call, a, b in out["graph"]:
            assert np.array_equal(a.view(np.uint32), _rank_order_sum(8191, world, call).view(np.uint32))
            assert np.array_equal(b.view(np.uint32), _rank_order_sum(16384, world, call).view(np.uint32))


def test_nccl_mode_keeps_nccl(cuda):
    outs = _run(cuda, 2, "nccl")
    for out in outs:
        assert not out["peer"]
        for count in (7, 16384):
            for call in range(3):
                assert np.allclose(out["eager"][count][call], _rank_order_sum(count, 2, call), rtol=1e-6, atol=2e-6)
