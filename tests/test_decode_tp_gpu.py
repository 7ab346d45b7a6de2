"""Tensor-parallel decoder (row split over 2, 4 or 8 GPUs, all-reduce after o
and down, the ranks' argmax candidates compared) against the same model at
TP=1.

Every exchange path is checked: the one-shot all-reduce over NVLink peer
memory (pushed from the o/down mat-vec's epilogue, or by a separate push
kernel where the mat-vec is not the team kernel), NCCL, and the persistent
step kernel (P100_DEC_STEP) with its own exchange.  Each rank initialises
its own slices from global coordinates, so TP=N holds the TP=1 model
exactly; the steps differ only in the summation order of the row-split
partial sums, so logits agree within the decoder bounds of
test_decode_gpu.py and the tokens agree where the top two logits are further
apart than the logit error.  One process per GPU; a case is skipped when the
box has fewer GPUs than ranks."""
import os
import socket

import numpy as np
import pytest

import p100_b200 as P
from test_decode_gpu import DECODE_LOGIT_TOL, TINY, mixed_types

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

SEED, NPOS, STEPS, TOKEN = 99, 100, 3, 7
# Per-tensor formats (five of them; a rank's Q6_K ffn_down slice has rows of
# 420 bytes, off the 16-byte grid) on a shape whose TP=2 slices are whole
# 256-value blocks.
SHAPES = {"tiny": TINY,
          "mixed": dict(TINY, hidden=512, n_head=8, n_head_kv=4, ffn=1024, tensor_types=mixed_types()),
          # splits 2, 4 and 8 ways: at TP=8 the o slice (k = 128) is not a team
          # mat-vec, so its exchange takes the separate push kernel
          "wide": dict(TINY, hidden=512, n_head=16, n_head_kv=8, ffn=2048)}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(dec):
    import torch
    dec.init_random(SEED)
    dec.fill_kv(NPOS, 5, 0.5)
    dec.set_state(NPOS, TOKEN)
    out = []
    for _ in range(STEPS):
        dec.step(1, torch.cuda.current_stream())
        pos, tok = dec.state()
        logits = dec.read(*dec.buffer(P.B_LOGITS)).view(np.float32).copy()
        out.append((pos, tok, logits))
    return out


def _rank(rank, world, port, q, allreduce, shape, flags):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      P100_TP_ALLREDUCE=allreduce)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    tp = dec = None
    try:
        box = [P.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = P.TP(box[0], world, rank, rank)
        dec = P.Decoder(P.LlamaConfig(**SHAPES[shape], flags=flags), tp)
        if flags == P.DEC_STEP:
            assert dec.path == P.DEC_PATH_STEP
        out = _run(dec)
        q.put((rank, dec.vocab_offset, [(p, t, l.tolist()) for p, t, l in out]))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))
    finally:
        if dec is not None:
            dec.close()   # releases the graph that holds the NCCL calls first
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


CASES = [(2, "tiny", "peer", 0), (2, "tiny", "nccl", 0), (2, "mixed", "peer", 0), (2, "mixed", "nccl", 0),
         (2, "wide", "peer", 0), (4, "wide", "peer", 0), (4, "wide", "nccl", 0), (8, "wide", "peer", 0),
         (8, "wide", "nccl", 0), (2, "wide", "peer", P.DEC_STEP), (4, "wide", "peer", P.DEC_STEP)]


@pytest.mark.parametrize("world,shape,allreduce,flags", CASES,
                         ids=[f"tp{w}-{s}-{a}{'-step' if f else ''}" for w, s, a, f in CASES])
def test_tpn_matches_tp1(cuda, world, shape, allreduce, flags):
    """allreduce: 'peer' = the one-shot all-reduce over NVLink peer memory
    (reduce inside the next RMSNorm), 'nccl' = ncclAllReduce; flags
    P100_DEC_STEP = the persistent step kernel."""
    if cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, allreduce, shape, flags)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    for r in res:
        assert r[1] != "error", r
    with cuda.cuda.device(0):
        dec = P.Decoder(P.LlamaConfig(**SHAPES[shape]))
        try:
            ref = _run(dec)
        finally:
            dec.close()
    for step in range(STEPS):
        pos1, tok1, logits1 = ref[step]
        full = np.zeros(SHAPES[shape]["vocab"], dtype=np.float32)
        for rank, off, out in res:
            pos, tok, logits = out[step]
            assert pos == pos1
            full[off:off + len(logits)] = logits
        assert all(r[2][step][1] == res[0][2][step][1] for r in res)   # every rank picks the same token
        err = np.max(np.abs(full - logits1))
        assert err <= DECODE_LOGIT_TOL * np.max(np.abs(logits1)), (step, err)
        top2 = np.sort(logits1)[-2:]
        if top2[1] - top2[0] > 2 * err:
            assert res[0][2][step][1] == tok1
        if res[0][2][step][1] != tok1:
            break   # the runs continue from different tokens: later steps are not comparable
