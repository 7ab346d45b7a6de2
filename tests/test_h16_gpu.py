"""The h16 activation path (p100_h16_prepare, p100_qmv_h16) on B200 against the
CPU restatement of qmv::prepare and qmv::h16_model (oracle/p100_oracle.cpp,
itself checked against the reference's evaluate().h8 / .h16).

The activation record is bit-exact.  A 32-block's value is bit-exact too (the
same HFMA2 chains, each product-and-add rounded once to fp16, then the same
FP32 operations); with k = 128 a row is one lane's four blocks added in
order, so Q4_0 and Q8_0 rows equal the model bit for bit.  Longer rows add
their 128-column ranges by a butterfly instead of the model's sequential
sum: within FP32 reassociation of the row."""
import numpy as np
import pytest

from conftest import QMV_NORM_TOL
from test_qmv_gpu import assert_qmv_close, dev, row_norms

import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu


def acts_of(orc, x):
    return np.concatenate([orc.prepare(xc) for xc in x])


@pytest.mark.parametrize("k,batch", [(32, 1), (4096, 2), (14336, 3)])
def test_h16_prepare_bit_exact(cuda, orc, k, batch):
    rng = np.random.default_rng(k + batch)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    x[0, :32] = 0.0                     # an all-zero block: scale 0, h 0
    if k > 64:
        x[0, 32:64] *= 1e-6             # tiny values: subnormal halves
    h, ss = P.h16_prepare(dev(cuda, x))
    a = acts_of(orc, x)
    gh = h.cpu().numpy().reshape(-1, 32)
    assert np.array_equal(gh.view(np.uint16), a["h"].astype(np.float16).view(np.uint16))
    gss = ss.cpu().numpy().reshape(-1, 2)
    assert np.array_equal(gss[:, 0].view(np.uint32), a["scale"].view(np.uint32))
    assert np.array_equal(gss[:, 1].view(np.uint32), a["sum"].view(np.uint32))


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0])
@pytest.mark.parametrize("chain", [8, 16])
def test_qmv_h16_one_lane_rows_bit_exact(cuda, orc, qtype, chain):
    """k = 128: every row is one lane's four blocks, added in the model's order;
    the weight rows come from the reference's own generator (random_row)."""
    k, rows, batch = 128, 300, 2
    w = orc.random_rows(qtype, k, rows, seed=61 + qtype)
    x = np.random.default_rng(5).standard_normal((batch, k)).astype(np.float32)
    h, ss = P.h16_prepare(dev(cuda, x))
    y = P.qmv_h16(qtype, dev(cuda, w), rows, k, h, ss, batch, chain).cpu().numpy()
    yref = orc.qmv_h16(qtype, w, rows, k, acts_of(orc, x), batch, chain)
    assert np.array_equal(y.view(np.uint32), yref.view(np.uint32))


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
@pytest.mark.parametrize("k,rows", [(256, 64), (4096, 1024), (14336, 512), (28672, 40)])
@pytest.mark.parametrize("chain", [8, 16])
def test_qmv_h16_matches_model(cuda, orc, qtype, k, rows, chain):
    w = W.weights(qtype, rows, k, seed=k + rows + qtype)
    x = W.activations(2, k, seed=k + 7)
    h, ss = P.h16_prepare(dev(cuda, x))
    y = P.qmv_h16(qtype, dev(cuda, w), rows, k, h, ss, 2, chain).cpu().numpy()
    yref = orc.qmv_h16(qtype, w, rows, k, acts_of(orc, x), 2, chain).astype(np.float64)
    err = assert_qmv_close(y, yref, row_norms(orc, qtype, w, rows, k), x, tol=QMV_NORM_TOL)
    assert err <= 1e-5, err   # FP32 reassociation of the row sum only
    assert P.device_error() == P.OK


def test_qmv_h16_rejects_shapes(cuda):
    w = cuda.zeros(4096, dtype=cuda.uint8, device="cuda")
    h = cuda.zeros(1024, dtype=cuda.float16, device="cuda")
    ss = cuda.zeros(64, device="cuda")
    y = cuda.zeros(8, device="cuda")
    with pytest.raises(P.P100Error):
        P.qmv_h16(P.Q4_0, w, 8, 96, h, ss, 1, 16, y=y)    # not a multiple of 128
    with pytest.raises(P.InvalidArgument):
        P.qmv_h16(P.Q4_0, w, 8, 128, h, ss, 1, 12, y=y)   # chain 8 or 16 only
    with pytest.raises(P.InvalidArgument):
        P.qmv_h16(P.Q4_K, w, 8, 128, h, ss, 1, 16, y=y)   # Q4_K: whole super-blocks
