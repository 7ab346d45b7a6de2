"""The batched mat-vec on the 5th-generation tensor cores (P100_QMV_TC:
tcgen05.mma kind::i8, operands and one accumulator per 32-value block in
tensor memory, weights by TMA), through the C-ABI.

Bar: within 1e-3 * ||w|| * ||x|| of prepare()+evaluate().q81 (the integer
block dots are exact; only the FP32 scaling order differs from the CPU
model), for Q4_0, Q8_0 and Q4_K; the same bar against the mma.sync kernel;
columns independent of the batch size; ragged row tiles (the TMA box reads
zeros past the last row) and K split over a cluster of CTAs."""
import numpy as np
import pytest

from test_qmv_gpu import assert_qmv_close, dev, q81_reference, row_norms

import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu
TYPES = [P.Q4_0, P.Q8_0, P.Q4_K]


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("k,rows,batch", [(4096, 14336, 16), (14336, 4096, 8), (4096, 1024, 5), (4096, 4096, 2),
                                          (256, 300, 3), (1024, 1000, 16), (8192, 130, 4)])
def test_tc_matches_q81_model(cuda, orc, qtype, k, rows, batch):
    w = W.weights(qtype, rows, k, seed=7 * k + rows + qtype)
    x = W.activations(batch, k, seed=k + batch)
    wd = dev(cuda, w)
    xq = P.q8_1_quantize(dev(cuda, x))
    y = P.qmv(qtype, wd, rows, k, xq, batch, flags=P.QMV_TC).cpu().numpy()
    wn = row_norms(orc, qtype, w, rows, k)
    if rows * k <= 4096 * 4096:
        assert_qmv_close(y, q81_reference(orc, qtype, w, rows, k, x).astype(np.float64), wn, x)
    # against the mma.sync kernel (itself checked against the model elsewhere)
    y_mma = P.qmv(qtype, wd, rows, k, xq, batch, flags=P.QMV_MMA).cpu().numpy()
    assert_qmv_close(y, y_mma.astype(np.float64), wn, x)
    assert P.device_error() == P.OK


@pytest.mark.parametrize("qtype", TYPES)
def test_tc_columns_independent(cuda, qtype):
    """A column's result does not depend on the other columns (batch 2..16
    pad the same 16-column tile with zeros)."""
    k, rows = 4096, 1024
    w = dev(cuda, W.weights(qtype, rows, k, seed=5 + qtype))
    xq = P.q8_1_quantize(dev(cuda, W.activations(16, k, seed=6)))
    full = P.qmv(qtype, w, rows, k, xq, 16, flags=P.QMV_TC).cpu().numpy()
    for batch in (2, 3, 9, 15):
        y = P.qmv(qtype, w, rows, k, xq, batch, flags=P.QMV_TC).cpu().numpy()
        assert np.array_equal(y, full[:batch]), batch


def test_tc_repeatable_and_chained(cuda):
    """Bit-identical repeats, and programmatic-dependent launches back to back."""
    k, rows = 14336, 4096
    w = dev(cuda, W.weights(P.Q4_0, rows, k, seed=3))
    xq = P.q8_1_quantize(dev(cuda, W.activations(8, k, seed=4)))
    a = P.qmv(P.Q4_0, w, rows, k, xq, 8, flags=P.QMV_TC).clone()
    y = cuda.empty(8, rows, device="cuda")
    for _ in range(5):
        P.qmv(P.Q4_0, w, rows, k, xq, 8, y=y, flags=P.QMV_TC | P.QMV_PDL)
    cuda.cuda.synchronize()
    assert cuda.equal(a, y)
    assert P.device_error() == P.OK
