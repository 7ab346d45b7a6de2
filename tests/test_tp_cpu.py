"""Row-split tensor parallelism, host side, on CPU: the split arithmetic, and a
two-rank gloo group that reproduces a full mat-vec from k-split partial sums
(the o/down exchange) and from row shards (q/k/v/gate/up), with the CPU oracle
standing in for the kernels.  Plus failure detection between ranks: a rank
that raises before the exchange makes its peer's collective fail within the
process-group timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from p100_b200 import tp as T
from p100_b200 import workloads as W


def test_split_range_and_errors():
    assert T.split_range(4096, 4, 1, 128) == (1024, 2048)
    with pytest.raises(ValueError):
        T.split_range(4096, 3, 0, 128)
    with pytest.raises(ValueError):
        T.split_range(10, 2, 2)


def test_llama70b_layer_split_tp8():
    s = T.LayerSplit(hidden=8192, n_head=64, n_kv_head=8, head_dim=128, ffn=28672, tp=8, rank=3)
    shapes = dict((n, (k, r)) for n, k, r in s.matvecs())
    assert shapes["q"] == (8192, 1024) and shapes["k"] == (8192, 128) and shapes["o"] == (1024, 8192)
    assert shapes["gate"] == (8192, 3584) and shapes["down"] == (3584, 8192)
    assert s.q_range() == (3072, 4096) and s.kv_range() == (384, 512) and s.allreduce_elems() == 16384
    with pytest.raises(ValueError):
        T.LayerSplit(hidden=4096, n_head=32, n_kv_head=8, head_dim=128, ffn=14336, tp=16, rank=0)


@pytest.mark.parametrize("qtype", [0, 1, 2])
def test_k_shard_blocks_match(orc, qtype):
    rows, k = 6, 1024
    w = W.weights(qtype, rows, k, seed=qtype)
    full = orc.dequantize(qtype, w, rows, k)
    a = T.k_shard(w, qtype, rows, k, 256, 768)
    assert np.array_equal(orc.dequantize(qtype, a, rows, 512), full[:, 256:768])
    r = T.row_shard(w, qtype, rows, k, 2, 5)
    assert np.array_equal(orc.dequantize(qtype, r, 3, k), full[2:5])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    import oracle
    orc = oracle.oracle()
    try:
        qtype, rows, k = 2, 96, 2048
        w = W.weights(qtype, rows, k, seed=11)
        x = W.activations(1, k, seed=12)[0]
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        # k split (o / down): partial sums, then one all-reduce
        k0, k1 = T.split_range(k, world, rank, 256)
        part = orc.qmv_q81(qtype, T.k_shard(w, qtype, rows, k, k0, k1), rows, k1 - k0,
                           orc.prepare(x[k0:k1]), 1)[0]
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        # row split (q/k/v/gate/up): each rank's rows, gathered
        r0, r1 = T.split_range(rows, world, rank)
        mine = torch.from_numpy(orc.qmv_q81(qtype, T.row_shard(w, qtype, rows, k, r0, r1), r1 - r0, k,
                                            orc.prepare(x), 1)[0].copy())
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        if rank == 0:
            out.put(("ok", t.numpy(), torch.cat(gathered).numpy()))
    except Exception as e:  # noqa: BLE001 — reported to the parent
        out.put(("error", rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _spawn(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    while not q.empty():
        results.append(q.get())
    return results


def test_two_rank_exchange_matches_full(orc):
    results = _spawn("ok")
    ok = [r for r in results if r[0] == "ok"]
    assert ok and not [r for r in results if r[0] == "error"], results
    _, summed, rows_cat = ok[0]
    qtype, rows, k = 2, 96, 2048
    w = W.weights(qtype, rows, k, seed=11)
    x = W.activations(1, k, seed=12)[0]
    full = orc.qmv_q81(qtype, w, rows, k, orc.prepare(x), 1)[0].astype(np.float64)
    deq = orc.dequantize(qtype, w, rows, k).astype(np.float64)
    norm = np.sqrt((deq ** 2).sum(1)) * np.sqrt((x.astype(np.float64) ** 2).sum())
    assert (np.abs(summed - full) / norm).max() <= 1e-5        # same block dots, re-associated sum
    assert np.array_equal(rows_cat, full.astype(np.float32))  # row shards are the full rows


def test_failed_rank_is_detected_not_hung():
    results = _spawn("fail")
    errors = {r[1]: r[2] for r in results if r[0] == "error"}
    assert 1 in errors and "fails before the exchange" in errors[1]
    # rank 0's collective ends with an error (peer gone) within the timeout
    assert 0 in errors
