"""The oracle's quantised mat-vec contract, pinned on CPU against the
reference: its golden qmv-numerics table byte for byte, its prepare() and
evaluate() outputs recorded in tests/golden/, and (where oracle/_ref exists)
the reference library itself on fresh seeded inputs."""
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, golden

import oracle


def test_golden_table_byte_for_byte(orc):
    """qmv_model.cpp restated reproduces tests/qmv_numerics.cpp's table."""
    exe = ROOT / "oracle" / "lib" / "qmv_table"
    if not exe.exists():
        oracle.build()
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert out == (GOLDEN / "qmv-numerics.txt").read_text()


def test_prepare_golden_bit_exact(orc):
    g = golden("q8_1.npz")
    for i, x in enumerate(g["x"]):
        acts = orc.prepare(x)
        assert np.array_equal(acts["qd"].view(np.uint32), g["qd"][i].view(np.uint32))
        assert np.array_equal(acts["qsum"].view(np.uint32), g["qsum"][i].view(np.uint32))
        assert np.array_equal(acts["q"].astype(np.int8), g["q"][i])


def test_q8_1_pack_layout(orc):
    x = np.linspace(-3, 5, 64, dtype=np.float32)
    acts = orc.prepare(x)
    packed = orc.pack_q8_1(acts)
    assert packed.size == 72
    for b in range(2):
        blk = packed[36 * b:36 * (b + 1)]
        assert blk[0:2].view(np.float16)[0] == np.float16(acts["qd"][b])
        assert blk[2:4].view(np.float16)[0] == np.float16(acts["qsum"][b])
        assert np.array_equal(blk[4:].view(np.int8), acts["q"][b].astype(np.int8))


def test_evaluate_golden(orc):
    g = golden("qmv.npz")
    for t, name in oracle.TYPE_NAMES.items():
        for k in (256, 4096, 14336):
            key = f"{name}_{k}"
            w, x = g[key + "_w"], g[key + "_x"]
            rows = g[key + "_wnorm"].size
            rb = w.size // rows
            for c in range(2):
                acts = orc.prepare(x[c])
                for r in range(rows):
                    e = orc.evaluate(t, w[r * rb:(r + 1) * rb], x[c], acts)
                    assert np.float32(e["q81"]).view(np.uint32) == g[key + "_q81"][c, r].view(np.uint32)
                    assert e["exact"] == g[key + "_exact"][c, r]
                    assert e["weight_norm"] == g[key + "_wnorm"][r]
            # the batched q81 entry point is the same sequential model
            acts = np.concatenate([orc.prepare(x[c]) for c in range(2)])
            y = orc.qmv_q81(t, w, rows, k, acts, 2)
            assert np.array_equal(y.view(np.uint32), g[key + "_q81"].view(np.uint32))


def _numpy_dequant(t, w, rows, k):
    """Independent numpy decode of the GGUF layouts (qmv_model.cpp:72-91,143)."""
    w = w.reshape(rows, -1)
    if t == oracle.Q4_0:
        b = w.reshape(rows, k // 32, 18)
        d = b[..., :2].copy().view(np.float16)[..., 0].astype(np.float64)
        qs = b[..., 2:].astype(np.int64)
        q = np.concatenate([qs & 15, qs >> 4], axis=-1) - 8
        return (d[..., None] * q).reshape(rows, k).astype(np.float32)
    if t == oracle.Q8_0:
        b = w.reshape(rows, k // 32, 34)
        d = b[..., :2].copy().view(np.float16)[..., 0].astype(np.float64)
        q = b[..., 2:].view(np.int8).astype(np.int64)
        return (d[..., None] * q).reshape(rows, k).astype(np.float32)
    b = w.reshape(rows, k // 256, 144)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    dmin = b[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float64)
    s = b[..., 4:16].astype(np.int64)
    qs = b[..., 16:].astype(np.int64)
    out = np.zeros((rows, k // 256, 8, 32))
    for j in range(8):
        if j < 4:
            sc, mn = s[..., j] & 63, s[..., j + 4] & 63
        else:
            sc = (s[..., j + 4] & 15) | ((s[..., j - 4] >> 6) << 4)
            mn = (s[..., j + 4] >> 4) | ((s[..., j] >> 6) << 4)
        q = (qs[..., (j // 2) * 32:(j // 2) * 32 + 32] >> ((j % 2) * 4)) & 15
        out[:, :, j, :] = (d * sc)[..., None] * q - (dmin * mn)[..., None]
    return out.reshape(rows, k).astype(np.float32)


@pytest.mark.parametrize("t", [oracle.Q4_0, oracle.Q8_0, oracle.Q4_K])
def test_dequantize_matches_numpy(orc, t):
    w = orc.random_rows(t, 1024, 9, 99 + t)
    got = orc.dequantize(t, w, 9, 1024)
    assert np.array_equal(got.view(np.uint32), _numpy_dequant(t, w, 9, 1024).view(np.uint32))


def test_shape_errors_use_reference_wording(orc):
    with pytest.raises(ValueError, match="whole activation blocks required"):
        orc.prepare(np.zeros(33, np.float32))
    with pytest.raises(ValueError, match="whole weight blocks required"):
        orc.random_rows(oracle.Q4_K, 128, 1, 1)


# ------------------------------------------------------------- against oracle/_ref
@pytest.mark.parametrize("t", [oracle.Q4_0, oracle.Q8_0, oracle.Q4_K])
def test_random_row_matches_reference(orc, ref, t):
    assert np.array_equal(orc.random_rows(t, 4096, 4, 1234 + t), ref.random_rows(t, 4096, 4, 1234 + t))


def test_prepare_matches_reference(orc, ref):
    rng = np.random.default_rng(11)
    for scale in (1e-7, 1e-3, 1.0, 3e3, 6e4):
        x = (rng.standard_normal(2048) * scale).astype(np.float32)
        x[64:96] = 0
        assert orc.prepare(x).tobytes() == ref.prepare(x).tobytes()


@pytest.mark.parametrize("t", [oracle.Q4_0, oracle.Q8_0, oracle.Q4_K])
def test_evaluate_matches_reference(orc, ref, t):
    rng = np.random.default_rng(100 + t)
    k = 2048
    w = ref.random_rows(t, k, 6, 555 + t)
    rb = w.size // 6
    for dist in range(3):
        x = rng.standard_normal(k).astype(np.float32) * (1000.0 if dist == 2 else 1.0)
        if dist == 1:
            x[rng.integers(0, k, 4)] *= 50
        acts = ref.prepare(x)
        for r in range(6):
            a = orc.evaluate(t, w[r * rb:(r + 1) * rb], x, acts)
            b = ref.evaluate(t, w[r * rb:(r + 1) * rb], x, acts)
            for field in a:
                assert np.asarray(a[field]).tobytes() == np.asarray(b[field]).tobytes(), field


@pytest.mark.parametrize("qtype", [0, 1, 2])
def test_h16_rows_equal_evaluate(orc, qtype):
    """p100o_qmv_h16 (the rows x columns h16 path the GPU tests compare with)
    is evaluate().h16 / .h8 row by row, bit for bit."""
    k, rows = 512, 6
    w = orc.random_rows(qtype, k, rows, 13 + qtype)
    x = np.random.default_rng(qtype).standard_normal((2, k)).astype(np.float32)
    acts = np.concatenate([orc.prepare(xc) for xc in x])
    rb = w.size // rows
    for chain, key in ((16, "h16"), (8, "h8")):
        y = orc.qmv_h16(qtype, w, rows, k, acts, 2, chain)
        for c in range(2):
            for r in range(rows):
                e = orc.evaluate(qtype, w[r * rb:(r + 1) * rb], x[c], orc.prepare(x[c]))
                assert np.float32(e[key]).view(np.uint32) == y[c, r].view(np.uint32)
