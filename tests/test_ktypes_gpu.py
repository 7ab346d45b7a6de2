"""ggml's Q5_K and Q6_K weights on B200 (p100_dequantize, p100_qmv: the team
kernel at batch 1 where a row is whole 16-byte units, the general mat-vec
kernel otherwise) against the CPU restatement (oracle/p100_oracle.cpp,
itself checked against ggml's dequantisation loops in
tests/test_oracle_ktypes.py).  Dequantisation is bit-exact; the mat-vec is
within the reference's normalised q81 tolerance of the oracle's q81 dot (and
of the exact FP64 dot)."""
import numpy as np
import pytest

from conftest import QMV_NORM_TOL
from test_qmv_gpu import assert_qmv_close, dev, q81_reference, row_norms

import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu
KTYPES = [P.Q5_K, P.Q6_K]


@pytest.mark.parametrize("qtype", KTYPES)
@pytest.mark.parametrize("rows,k", [(7, 256), (300, 4096), (64, 14336)])
def test_dequantize_bit_exact(cuda, orc, qtype, rows, k):
    w = W.weights(qtype, rows, k, seed=rows + k + qtype)
    got = P.dequantize(qtype, dev(cuda, w), rows, k).cpu().numpy()
    want = orc.dequantize(qtype, w, rows, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype", KTYPES)
@pytest.mark.parametrize("rows,k,batch", [(1024, 4096, 1), (333, 4096, 3), (256, 14336, 16), (40, 256, 2)])
def test_qmv_within_tolerance(cuda, orc, qtype, rows, k, batch):
    w = W.weights(qtype, rows, k, seed=11 * qtype + k)
    x = W.activations(batch, k, seed=k + batch)
    xq = P.q8_1_quantize(dev(cuda, x))
    y = P.qmv(qtype, dev(cuda, w), rows, k, xq, batch).cpu().numpy()
    wn = row_norms(orc, qtype, w, rows, k)
    err = assert_qmv_close(y, q81_reference(orc, qtype, w, rows, k, x).astype(np.float64), wn, x)
    assert err <= 1e-5, err   # the same slab arithmetic, summed in another order
    exact = x.astype(np.float64) @ orc.dequantize(qtype, w, rows, k).astype(np.float64).T
    assert_qmv_close(y, exact, wn, x, tol=QMV_NORM_TOL)
    assert P.device_error() == P.OK


# Batch 1 on the team kernel: k = 4096 / 8192 / 14336 / 28672 (compiled
# group counts 16, 32, 56, 112; teams of 16 and 32 lanes, of 2 and 4 warps),
# 6144 (the runtime-shaped variant), row counts that leave a partial last
# stage; Q6_K rows that are not whole 16-byte units (k = 7168 and 3584, the
# down slices of tensor parallelism 2 and 4; k = 1280: 1050-byte rows), whose
# stages start off the 16-byte grid; and a shape that falls back to the
# general kernel (33 Q6_K rows of 1050 bytes do not end on the grid).
@pytest.mark.parametrize("qtype", KTYPES)
@pytest.mark.parametrize("rows,k", [(4099, 4096), (1000, 8192), (777, 14336), (301, 28672), (515, 6144),
                                    (20000, 4096), (4096, 7168), (1000, 3584), (40, 1280), (33, 1280)])
def test_qmv_batch1_team_kernel(cuda, orc, qtype, rows, k):
    w = W.weights(qtype, rows, k, seed=5 * qtype + rows)
    x = W.activations(1, k, seed=rows)
    xq = P.q8_1_quantize(dev(cuda, x))
    y = P.qmv(qtype, dev(cuda, w), rows, k, xq, 1).cpu().numpy()
    wn = row_norms(orc, qtype, w, rows, k)
    err = assert_qmv_close(y, q81_reference(orc, qtype, w, rows, k, x).astype(np.float64), wn, x)
    assert err <= 1e-5, err
    assert P.device_error() == P.OK


@pytest.mark.parametrize("qtype", KTYPES)
def test_h16_and_whole_blocks(cuda, qtype):
    w = cuda.zeros(1 << 16, dtype=cuda.uint8, device="cuda")
    h = cuda.zeros(4096, dtype=cuda.float16, device="cuda")
    ss = cuda.zeros(512, device="cuda")
    y = cuda.zeros(64, device="cuda")
    with pytest.raises(P.P100Error) as e:
        P.qmv_h16(qtype, w, 8, 256, h, ss, 1, 16, y=y)
    assert e.value.status == P.ERR_UNSUPPORTED
    xq = cuda.zeros(4096, dtype=cuda.uint8, device="cuda")
    with pytest.raises(P.InvalidArgument):
        P.qmv(qtype, w, 8, 128, xq, 1, y=y)     # a super-block is 256 values


@pytest.mark.parametrize("qtype", KTYPES)
@pytest.mark.parametrize("rows,k,batch", [(4096, 4096, 2), (515, 14336, 5), (40, 1280, 16), (33, 1280, 3)])
def test_qmv_batches_equal_columns(cuda, orc, qtype, rows, k, batch):
    """Batch 2..16 of Q5_K / Q6_K: one team-kernel launch per column where the
    team kernel takes the matrix (the general kernel for 33 Q6_K rows of 1050
    bytes), the bits of batch-1 calls column by column, and within the q81
    tolerance of the oracle."""
    w = dev(cuda, W.weights(qtype, rows, k, seed=7 * qtype + rows))
    x = W.activations(batch, k, seed=batch + k)
    xq = P.q8_1_quantize(dev(cuda, x))
    y = P.qmv(qtype, w, rows, k, xq, batch).cpu().numpy()
    cb = P.q8_1_bytes(k, 1)
    for c in range(batch):
        yc = P.qmv(qtype, w, rows, k, xq[c * cb:(c + 1) * cb], 1).cpu().numpy()
        assert np.array_equal(y[c].view(np.uint32), yc[0].view(np.uint32)), c
    wh = w.cpu().numpy()
    err = assert_qmv_close(y, q81_reference(orc, qtype, wh, rows, k, x).astype(np.float64),
                           row_norms(orc, qtype, wh, rows, k), x)
    assert err <= 1e-5, err
    assert P.device_error() == P.OK
