"""Row-split tensor-parallel layout for the quantised decode path.

Megatron-style split of a transformer layer over N GPUs of one box, the
layout that replaces the reference's two-GPU PCIe split (src/p2p/p2p.cpp,
bench/phase0.sh:148-164):

* column-parallel (split by output rows, whole heads): q, k, v, gate, up —
  each rank computes its own slice of the outputs; nothing is exchanged;
* row-parallel (split along k): o and down — each rank multiplies its k slice
  by the matching slice of its activations and the ranks' partial outputs
  are summed by one fp32 all-reduce of the hidden vector (p100_tp_allreduce_sum);
* the LM head is split by vocabulary rows; RMSNorm and the residual stream are
  replicated.

Q8_1 activation blocks cover 32 values and weight blocks 32 (Q4_0/Q8_0) or
256 (Q4_K) values, so every k split falls on a Q4_K super-block boundary:
a k slice of the activations quantises to exactly the blocks the full row
would give, and every rank's integer block dots are those of the full matrix.
"""
from __future__ import annotations

from dataclasses import dataclass

BLOCK_ELEMS = {0: 32, 1: 32, 2: 256, 3: 256, 4: 256}
BLOCK_BYTES = {0: 18, 1: 34, 2: 144, 3: 176, 4: 210}


def split_range(total, parts, rank, align=1):
    """[lo, hi) of rank's equal share of `total`, in units of `align`."""
    if parts < 1 or not 0 <= rank < parts:
        raise ValueError(f"rank {rank} of {parts}")
    if total % (parts * align):
        raise ValueError(f"{total} does not split into {parts} shares of whole {align}-element units")
    share = total // parts
    return rank * share, (rank + 1) * share


def row_shard(w, qtype, rows, k, r0, r1):
    """Rows r0..r1 of a row-major block matrix (a contiguous slice)."""
    rb = k // BLOCK_ELEMS[qtype] * BLOCK_BYTES[qtype]
    return w[r0 * rb:r1 * rb]


def k_shard(w, qtype, rows, k, k0, k1):
    """Columns k0..k1 (whole blocks) of every row, as a new row-major matrix."""
    be, bb = BLOCK_ELEMS[qtype], BLOCK_BYTES[qtype]
    if k0 % be or k1 % be:
        raise ValueError("k split must fall on block boundaries")
    rb = k // be * bb
    view = w.reshape(rows, rb)
    return view[:, k0 // be * bb:k1 // be * bb].reshape(-1)


@dataclass(frozen=True)
class LayerSplit:
    """Per-rank shapes of one decoder layer under row-split TP."""
    hidden: int
    n_head: int
    n_kv_head: int
    head_dim: int
    ffn: int
    tp: int
    rank: int

    def __post_init__(self):
        if self.n_head % self.tp or self.n_kv_head % self.tp:
            raise ValueError("heads must divide evenly over the TP ranks")
        if self.ffn % (self.tp * 256) or (self.n_head * self.head_dim) % (self.tp * 256):
            raise ValueError("row-parallel k slices must be whole Q4_K super-blocks")

    @property
    def q_rows(self):
        return self.n_head // self.tp * self.head_dim

    @property
    def kv_rows(self):
        return self.n_kv_head // self.tp * self.head_dim

    @property
    def ffn_rows(self):
        return self.ffn // self.tp

    def q_range(self):
        return split_range(self.n_head * self.head_dim, self.tp, self.rank, self.head_dim)

    def kv_range(self):
        return split_range(self.n_kv_head * self.head_dim, self.tp, self.rank, self.head_dim)

    def ffn_range(self):
        return split_range(self.ffn, self.tp, self.rank, 256)

    def matvecs(self):
        """(name, k, rows) of every per-rank mat-vec of the layer, in order."""
        return [("q", self.hidden, self.q_rows), ("k", self.hidden, self.kv_rows), ("v", self.hidden, self.kv_rows),
                ("o", self.q_rows, self.hidden), ("gate", self.hidden, self.ffn_rows),
                ("up", self.hidden, self.ffn_rows), ("down", self.ffn_rows, self.hidden)]

    def allreduce_elems(self):
        """fp32 elements summed per layer: the o and down outputs."""
        return 2 * self.hidden if self.tp > 1 else 0
