"""GPU parity of the quantised mat-vec path through the C-ABI.

Bar: Q8_1 activation blocks and dequantised weights bit-exact with the CPU
contract; mat-vec within 1e-3 * ||w|| * ||x|| of prepare()+evaluate().q81
(tests/h2_mmv_gpu.cu:89,141 use the same normalisation)."""
import numpy as np
import pytest

from conftest import QMV_NORM_TOL, golden

import oracle
import p100_b200 as P
from p100_b200 import workloads as W

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def q81_reference(orc, qtype, w, rows, k, x):
    acts = np.concatenate([orc.prepare(xc) for xc in x])
    y, _ = orc.qmv_q81_threaded(qtype, w, rows, k, acts, x.shape[0], oracle.host_cores())
    return y


def row_norms(orc, qtype, w, rows, k):
    rb = w.size // rows
    out = np.empty(rows)
    for r0 in range(0, rows, 1024):
        r1 = min(rows, r0 + 1024)
        deq = orc.dequantize(qtype, w[r0 * rb:r1 * rb], r1 - r0, k).astype(np.float64)
        out[r0:r1] = np.sqrt((deq * deq).sum(axis=1))
    return out


def assert_qmv_close(y, yref, wn, x, tol=QMV_NORM_TOL):
    xn = np.sqrt((x.astype(np.float64) ** 2).sum(axis=1))
    err = np.abs(y.astype(np.float64) - yref) / (wn[None, :] * xn[:, None] + 1e-30)
    assert err.max() <= tol, f"max normalised error {err.max():.3e}"
    return err.max()


# ------------------------------------------------------------------ Q8_1
def test_q8_1_bit_exact_golden(cuda, orc):
    g = golden("q8_1.npz")
    for i, x in enumerate(g["x"]):
        got = P.q8_1_quantize(dev(cuda, x)).cpu().numpy()
        blocks = got.reshape(-1, 36)
        assert np.array_equal(blocks[:, 0:2].copy().view(np.uint16)[:, 0],
                              g["qd"][i].astype(np.float16).view(np.uint16))
        assert np.array_equal(blocks[:, 2:4].copy().view(np.uint16)[:, 0],
                              g["qsum"][i].astype(np.float16).view(np.uint16))
        assert np.array_equal(blocks[:, 4:].view(np.int8), g["q"][i])


@pytest.mark.parametrize("k,batch", [(32, 1), (4096, 3), (14336, 16), (28672, 2)])
def test_q8_1_bit_exact_random(cuda, orc, k, batch):
    rng = np.random.default_rng(k + batch)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    x[0, :32] = 0
    x[-1] *= rng.standard_normal(k).astype(np.float32) * 3
    if batch > 2:
        x[1] *= 1e4
        x[2] *= 1e-5
    got = P.q8_1_quantize(dev(cuda, x)).cpu().numpy()
    assert np.array_equal(got, orc.quantize_q8_1(x, k))


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
@pytest.mark.parametrize("k", [256, 4096])
def test_dequantize_bit_exact(cuda, orc, qtype, k):
    rows = 19
    w = orc.random_rows(qtype, k, rows, 3 + qtype + k)
    got = P.dequantize(qtype, dev(cuda, w), rows, k).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), orc.dequantize(qtype, w, rows, k).view(np.uint32))


# ------------------------------------------------------------------ mat-vec
def test_qmv_golden(cuda, orc):
    g = golden("qmv.npz")
    for qtype, name in oracle.TYPE_NAMES.items():
        for k in (256, 4096, 14336):
            key = f"{name}_{k}"
            w, x = g[key + "_w"], g[key + "_x"]
            rows = g[key + "_wnorm"].size
            xq = P.q8_1_quantize(dev(cuda, x))
            y = P.qmv(qtype, dev(cuda, w), rows, k, xq, batch=2).cpu().numpy()
            assert_qmv_close(y, g[key + "_q81"].astype(np.float64), g[key + "_wnorm"], x)
            # and it tracks the exact FP64 dot like the CPU q81 model does
            xn = np.sqrt((x.astype(np.float64) ** 2).sum(axis=1))
            e_gpu = np.abs(y - g[key + "_exact"]) / (g[key + "_wnorm"][None] * xn[:, None])
            e_cpu = np.abs(g[key + "_q81"] - g[key + "_exact"]) / (g[key + "_wnorm"][None] * xn[:, None])
            assert e_gpu.max() <= e_cpu.max() + QMV_NORM_TOL


SHAPES = [(k, rows) for _, k, rows in W.LLAMA3_8B_SHAPES]


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
@pytest.mark.parametrize("k,rows", SHAPES)
def test_qmv_llama_shapes(cuda, orc, qtype, k, rows):
    """Config-2 shapes at batch 1 and 4 against the sequential CPU model
    (batch 4: the default kernel choice, and the mma.sync kernel forced)."""
    w = W.weights(qtype, rows, k, seed=1000 + k + rows + qtype)
    x = W.activations(4, k, seed=77 + k)
    wd = dev(cuda, w)
    wn = row_norms(orc, qtype, w, rows, k)
    yref = q81_reference(orc, qtype, w, rows, k, x).astype(np.float64)
    xq = P.q8_1_quantize(dev(cuda, x))
    for flags in (0, P.QMV_MMA):
        y4 = P.qmv(qtype, wd, rows, k, xq, batch=4, flags=flags).cpu().numpy()
        assert_qmv_close(y4, yref, wn, x)
    y1 = P.qmv(qtype, wd, rows, k, xq[: k // 32 * 36], batch=1).cpu().numpy()
    assert_qmv_close(y1, yref[:1], wn, x[:1])


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
def test_qmv_batch_columns_independent(cuda, orc, qtype):
    """A column's result does not depend on the other columns: batch sizes
    2..16 (one kernel family) give bit-identical columns, and the batch-1
    kernel agrees with them to FP32 reassociation error."""
    k, rows = 4096, 1024
    wh = W.weights(qtype, rows, k, seed=5 + qtype)
    w = dev(cuda, wh)
    x = W.activations(16, k, seed=6)
    xq = P.q8_1_quantize(dev(cuda, x))
    nbytes = k // 32 * 36
    full = P.qmv(qtype, w, rows, k, xq, 16).cpu().numpy()
    for batch in (2, 3, 5, 8, 13):
        y = P.qmv(qtype, w, rows, k, xq, batch).cpu().numpy()
        assert np.array_equal(y, full[:batch]), batch
    wn = row_norms(orc, qtype, wh, rows, k)
    for c in range(16):
        single = P.qmv(qtype, w, rows, k, xq[c * nbytes:(c + 1) * nbytes], 1).cpu().numpy()
        assert_qmv_close(single, full[c:c + 1].astype(np.float64), wn, x[c:c + 1], tol=1e-6)


def test_qmv_batch16_full_shape(cuda, orc):
    """Batch 16 on the down projection against the CPU model."""
    k, rows = 14336, 4096
    w = W.weights(P.Q4_0, rows, k, seed=99)
    x = W.activations(16, k, seed=98)
    yref = q81_reference(orc, P.Q4_0, w, rows, k, x).astype(np.float64)
    y = P.qmv(P.Q4_0, dev(cuda, w), rows, k, P.q8_1_quantize(dev(cuda, x)), 16).cpu().numpy()
    assert_qmv_close(y, yref, row_norms(orc, P.Q4_0, w, rows, k), x)


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
@pytest.mark.parametrize("k,rows,offset", [(256, 1, 0), (256, 17, 0), (512, 300, 2), (8192, 33, 0),
                                            (28672, 40, 0), (1024, 5, 18)])
def test_qmv_edge_shapes(cuda, orc, qtype, k, rows, offset):
    """Tiny and ragged shapes, 2-byte-aligned weights (generic kernel), k up to 28672."""
    if k % P.BLOCK_ELEMS[qtype]:
        pytest.skip("not whole blocks")
    w = W.weights(qtype, rows, k, seed=k + rows + qtype)
    x = W.activations(3, k, seed=k)
    x[1, :64] = 0
    buf = cuda.zeros(w.size + offset, dtype=cuda.uint8, device="cuda")
    buf[offset:] = dev(cuda, w)
    y = P.qmv(qtype, buf[offset:], rows, k, P.q8_1_quantize(dev(cuda, x)), 3).cpu().numpy()
    assert_qmv_close(y, q81_reference(orc, qtype, w, rows, k, x).astype(np.float64),
                     row_norms(orc, qtype, w, rows, k), x)


@pytest.mark.parametrize("qtype", [P.Q4_0, P.Q8_0, P.Q4_K])
@pytest.mark.parametrize("k,rows", [(256, 7), (768, 150), (4096, 301), (8192, 97), (12288, 65), (14336, 45),
                                    (28672, 23)])
def test_qmv_team_batch1_shapes(cuda, orc, qtype, k, rows):
    """Batch 1 on 16-byte-aligned buffers (the team kernel): the group counts
    compiled in (k = 4096, 8192, 14336, 28672), runtime-shaped ones (256, 768,
    12288 whose team spans two warps), and row counts that leave a ragged
    last stage."""
    w = W.weights(qtype, rows, k, seed=31 * k + rows + qtype)
    x = W.activations(1, k, seed=k + 5)
    y = P.qmv(qtype, dev(cuda, w), rows, k, P.q8_1_quantize(dev(cuda, x)), 1).cpu().numpy()
    assert_qmv_close(y, q81_reference(orc, qtype, w, rows, k, x).astype(np.float64),
                     row_norms(orc, qtype, w, rows, k), x)


def test_qmv_k32_generic(cuda, orc):
    for qtype in (P.Q4_0, P.Q8_0):
        w = orc.random_rows(qtype, 32, 9, 4)
        x = W.activations(2, 32, seed=3)
        y = P.qmv(qtype, dev(cuda, w), 9, 32, P.q8_1_quantize(dev(cuda, x)), 2).cpu().numpy()
        assert_qmv_close(y, q81_reference(orc, qtype, w, 9, 32, x).astype(np.float64),
                         row_norms(orc, qtype, w, 9, 32), x)


def test_qmv_zero_activation_and_rows(cuda):
    k, rows = 4096, 64
    w = dev(cuda, W.weights(P.Q4_0, rows, k, seed=1))
    xq = P.q8_1_quantize(cuda.zeros(1, k, device="cuda"))
    assert cuda.count_nonzero(P.qmv(P.Q4_0, w, rows, k, xq, 1)).item() == 0
    y = cuda.full((1, 1), 7.0, device="cuda")
    P.qmv(P.Q4_0, w, 0, k, xq, 1, y=y)   # rows == 0: nothing written
    assert y.item() == 7.0


def test_qmv_deterministic_and_pdl(cuda):
    k, rows = 14336, 4096
    w = dev(cuda, W.weights(P.Q4_K, rows, k, seed=2))
    x = dev(cuda, W.activations(2, k, seed=3))
    xq = P.q8_1_quantize(x)
    a = P.qmv(P.Q4_K, w, rows, k, xq, 2).clone()
    for _ in range(3):
        xq = P.q8_1_quantize(x)                        # producer kernel right before
        b = P.qmv(P.Q4_K, w, rows, k, xq, 2, flags=P.QMV_PDL)
        assert cuda.equal(a, b)
    assert P.device_error() == P.OK


def test_qmv_invalid_arguments(cuda):
    w = cuda.zeros(1000, dtype=cuda.uint8, device="cuda")
    xq = cuda.zeros(1000, dtype=cuda.uint8, device="cuda")
    with pytest.raises(P.InvalidArgument, match="whole weight blocks required"):
        P.qmv(P.Q4_K, w, 1, 128, xq, 1)
    with pytest.raises(P.InvalidArgument, match="batch"):
        P.qmv(P.Q4_0, w, 1, 32, xq, 17)
    with pytest.raises(P.InvalidArgument, match="unknown weight type"):
        P.qmv(7, w, 1, 32, xq, 1)
    with pytest.raises(P.InvalidArgument, match="exclude each other"):
        P.qmv(P.Q4_0, w, 1, 32, xq, 2, flags=P.QMV_TC | P.QMV_MMA)


# ------------------------------------------------- fp32 activations
@pytest.mark.parametrize("qtype", [W.Q4_0, W.Q8_0, W.Q4_K, W.Q5_K, W.Q6_K])
@pytest.mark.parametrize("rows,k", [(4096, 4096), (1031, 14336), (333, 6144), (257, 28672), (64, 256), (63, 256)])
def test_qmv_f32_equals_quantize_then_qmv(cuda, qtype, rows, k):
    """p100_qmv_f32 gives the bits of p100_q8_1_quantize followed by p100_qmv,
    on two calls in a row: with scratch (the quantiser then the mat-vec as
    its programmatic dependent; the scratch holds the Q8_1 row) and without
    (the quantisation fused into the team kernel; 63 Q6_K rows of 210 bytes
    end off the 16-byte grid, which that kernel does not take: refused)."""
    w = dev(cuda, W.weights(qtype, rows, k, seed=rows + k + qtype))
    x = dev(cuda, W.activations(1, k, seed=k + qtype))
    xq = P.q8_1_quantize(x)
    want = P.qmv(qtype, w, rows, k, xq, 1).cpu().numpy()
    scratch = cuda.full((P.q8_1_bytes(k, 1),), 7, dtype=cuda.uint8, device="cuda")
    for flags in (0, P.QMV_PDL):
        got = P.qmv_f32(qtype, w, rows, k, x, x_q8_1=scratch, flags=flags).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert np.array_equal(scratch.cpu().numpy(), xq.cpu().numpy())
    if qtype == W.Q6_K and rows * (k // 256 * 210) % 16:
        with pytest.raises(P.P100Error) as e:
            P.qmv_f32(qtype, w, rows, k, x)
        assert e.value.status == P.ERR_UNSUPPORTED
    else:
        for flags in (0, P.QMV_PDL):
            got = P.qmv_f32(qtype, w, rows, k, x, flags=flags).cpu().numpy()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert P.device_error() == P.OK


def test_qmv_f32_batches_and_rejections(cuda):
    k, rows, b = 4096, 500, 4
    w = dev(cuda, W.weights(W.Q4_0, rows, k, seed=3))
    x = dev(cuda, W.activations(b, k, seed=4))
    want = P.qmv(W.Q4_0, w, rows, k, P.q8_1_quantize(x), b).cpu().numpy()
    scratch = cuda.empty(P.q8_1_bytes(k, b), dtype=cuda.uint8, device="cuda")
    got = P.qmv_f32(W.Q4_0, w, rows, k, x, batch=b, x_q8_1=scratch).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    with pytest.raises(P.P100Error) as e:          # batch 4 without scratch
        P.qmv_f32(W.Q4_0, w, rows, k, x, batch=b)
    assert e.value.status == P.ERR_UNSUPPORTED
    xs = cuda.zeros(k + 1, device="cuda")[1:]       # 4-byte aligned only: not fused
    with pytest.raises(P.P100Error) as e:
        P.qmv_f32(W.Q4_0, w, rows, k, xs)
    assert e.value.status == P.ERR_UNSUPPORTED
    with pytest.raises(P.InvalidArgument):
        P.qmv_f32(W.Q4_0, w, rows, k, x[:1], flags=8)
    with pytest.raises(P.InvalidArgument):
        P.q8_1_quantize(x, flags=8)
