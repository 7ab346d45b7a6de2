"""GGUF files (p100_b200/gguf.py) on CPU: the writer and reader agree on
every metadata type, tensor bytes and the data alignment; a llama file
yields the decoder configuration and each matrix's format (files that mix
formats, as llama.cpp's Q4_K_M files do, included); malformed files and
matrices in formats the decoder does not read are rejected with the
reason."""
import struct

import numpy as np
import pytest

from p100_b200 import gguf
from p100_b200 import workloads as W

TINY = dict(n_layer=2, hidden=256, n_head=4, n_head_kv=2, head_dim=64, ffn=512, vocab=300)


def llama_tensors(qtype, seed=0, tied=False, **shape):
    """A llama tensor list in llama.cpp's names for a random model."""
    s = dict(TINY, **shape)
    H, hd, F, V = s["hidden"], s["head_dim"], s["ffn"], s["vocab"]
    nq, nkv = s["n_head"], s["n_head_kv"]
    gt = gguf.GGML_OF_P100[qtype]
    rng = np.random.default_rng(seed)
    norm = lambda: (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    w = lambda rows, k, i: W.weights(qtype, rows, k, seed=seed * 100 + i)
    t = [("token_embd.weight", gt, (H, V), w(V, H, 1)), ("output_norm.weight", gguf.GGML_F32, (H,), norm())]
    if not tied:
        t.append(("output.weight", gt, (H, V), w(V, H, 2)))
    for l in range(s["n_layer"]):
        b = f"blk.{l}."
        t += [(b + "attn_norm.weight", gguf.GGML_F32, (H,), norm()),
              (b + "attn_q.weight", gt, (H, nq * hd), w(nq * hd, H, 10 * l + 3)),
              (b + "attn_k.weight", gt, (H, nkv * hd), w(nkv * hd, H, 10 * l + 4)),
              (b + "attn_v.weight", gt, (H, nkv * hd), w(nkv * hd, H, 10 * l + 5)),
              (b + "attn_output.weight", gt, (nq * hd, H), w(H, nq * hd, 10 * l + 6)),
              (b + "ffn_norm.weight", gguf.GGML_F32, (H,), norm()),
              (b + "ffn_gate.weight", gt, (H, F), w(F, H, 10 * l + 7)),
              (b + "ffn_up.weight", gt, (H, F), w(F, H, 10 * l + 8)),
              (b + "ffn_down.weight", gt, (F, H), w(H, F, 10 * l + 9))]
    meta = {"general.architecture": "llama", "llama.block_count": s["n_layer"], "llama.embedding_length": H,
            "llama.attention.head_count": nq, "llama.attention.head_count_kv": nkv,
            "llama.feed_forward_length": F, "llama.context_length": 8192, "llama.rope.freq_base": 500000.0,
            "llama.attention.layer_norm_rms_epsilon": 1e-5, "llama.rope.dimension_count": hd,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(V)]}
    return meta, t


def test_round_trip(tmp_path):
    meta = {"a.u32": 7, "a.i64": -5, "a.f32": 1.5, "a.str": "héllo", "a.bool": True,
            "a.arr_f32": np.arange(5, dtype=np.float32), "a.arr_i32": np.array([1, -2], dtype=np.int32),
            "a.strs": ["x", "yz", ""]}
    w = W.weights(W.Q4_K, 3, 512, seed=1)
    v = np.arange(96, dtype=np.float32)
    tensors = [("w", gguf.GGML_Q4_K, (512, 3), w), ("v", gguf.GGML_F32, (96,), v),
               ("h", gguf.GGML_F16, (8, 2), np.arange(16, dtype=np.float16))]
    p = tmp_path / "m.gguf"
    gguf.write_gguf(p, meta, tensors, alignment=64)
    with gguf.GGUFFile(str(p)) as g:
        assert g.version == 3 and g.data_offset % 64 == 0
        assert g.metadata["a.u32"] == 7 and g.metadata["a.i64"] == -5 and g.metadata["a.f32"] == 1.5
        assert g.metadata["a.str"] == "héllo" and g.metadata["a.bool"] is True
        assert np.array_equal(g.metadata["a.arr_f32"], meta["a.arr_f32"])
        assert np.array_equal(g.metadata["a.arr_i32"], meta["a.arr_i32"])
        assert g.metadata["a.strs"] == ["x", "yz", ""] and g.metadata["general.alignment"] == 64
        assert all(t.offset % 64 == 0 for t in g.tensors.values())
        assert np.array_equal(g.tensor_bytes("w"), w)
        assert np.array_equal(g.tensor_bytes("v").view(np.float32), v)
        assert g.tensors["w"].dims == (512, 3) and g.tensors["w"].ggml_type == gguf.GGML_Q4_K


@pytest.mark.parametrize("qtype", [W.Q4_0, W.Q8_0, W.Q4_K])
def test_llama_config(tmp_path, qtype):
    meta, t = llama_tensors(qtype, hidden=512, n_head=8, head_dim=64, tied=qtype == W.Q8_0)
    p = tmp_path / "llama.gguf"
    gguf.write_gguf(p, meta, t)
    with gguf.GGUFFile(str(p)) as g:
        cfg, wt = gguf.llama_config(g, max_ctx=1024)
        assert cfg == dict(n_layer=2, hidden=512, n_head=8, n_head_kv=2, head_dim=64, ffn=512, vocab=300,
                           max_ctx=1024, rope_theta=500000.0, norm_eps=pytest.approx(1e-5), wtype=qtype, flags=0,
                           kv_type=0)
        lm, types = gguf.llama_tensors(g, cfg)
        assert lm == ("token_embd.weight" if qtype == W.Q8_0 else "output.weight")
        assert wt == gguf.GGML_OF_P100[qtype] and types == [qtype] * (2 + 7 * 2)


def test_rejections(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(gguf.GGUFError, match="not a GGUF"):
        gguf.GGUFFile(str(p))
    meta, t = llama_tensors(W.Q4_0)
    gguf.write_gguf(p, meta, t)
    data = p.read_bytes()
    (tmp_path / "cut.gguf").write_bytes(data[:len(data) // 2])
    with pytest.raises(gguf.GGUFError, match="past the end|truncated"):
        gguf.GGUFFile(str(tmp_path / "cut.gguf"))
    # a matrix in a format the mat-vec does not read (F16)
    meta, t = llama_tensors(W.Q4_K)
    t = [(n, gguf.GGML_F16, d, np.zeros(d[0] * d[1], np.float16)) if n == "blk.1.ffn_down.weight"
         else (n, gt, d, x) for n, gt, d, x in t]
    gguf.write_gguf(p, meta, t)
    with gguf.GGUFFile(str(p)) as g:
        cfg, wt = gguf.llama_config(g)
        with pytest.raises(gguf.GGUFError, match="blk.1.ffn_down.weight is F16"):
            gguf.llama_tensors(g, cfg)
    meta["general.architecture"] = "qwen2"
    gguf.write_gguf(p, meta, t)
    with gguf.GGUFFile(str(p)) as g, pytest.raises(gguf.GGUFError, match="architecture"):
        gguf.llama_config(g)


def test_mixed_formats(tmp_path):
    """A Q4_K_M-style file: Q4_K, with attn_v and ffn_down of layer 1 and the
    output matrix in Q6_K and one ffn_up in Q5_K: each matrix's format lands
    at its tensor_types index."""
    meta, t = llama_tensors(W.Q4_K)
    swap = {"blk.1.attn_v.weight": W.Q6_K, "blk.1.ffn_down.weight": W.Q6_K, "output.weight": W.Q6_K,
            "blk.0.ffn_up.weight": W.Q5_K}
    t = [(n, gguf.GGML_OF_P100[swap[n]], d, W.weights(swap[n], d[1], d[0], seed=5)) if n in swap
         else (n, gt, d, x) for n, gt, d, x in t]
    p = tmp_path / "mixed.gguf"
    gguf.write_gguf(p, meta, t)
    with gguf.GGUFFile(str(p)) as g:
        cfg, wt = gguf.llama_config(g)
        assert wt == gguf.GGML_Q4_K and cfg["wtype"] == W.Q4_K
        lm, types = gguf.llama_tensors(g, cfg)
    want = [W.Q4_K] * (2 + 7 * 2)
    want[1] = W.Q6_K                                           # output
    want[2 + 7 * 0 + gguf.LAYER_MATRICES.index("ffn_up")] = W.Q5_K
    want[2 + 7 * 1 + gguf.LAYER_MATRICES.index("attn_v")] = W.Q6_K
    want[2 + 7 * 1 + gguf.LAYER_MATRICES.index("ffn_down")] = W.Q6_K
    assert lm == "output.weight" and types == want


def test_tp_shards_of_k_quants():
    """Row and K slices of Q5_K / Q6_K matrices fall on their 256-value blocks."""
    from p100_b200 import tp
    for qt, bb in ((W.Q5_K, 176), (W.Q6_K, 210)):
        w = W.weights(qt, 4, 1024, seed=2)
        assert tp.row_shard(w, qt, 4, 1024, 1, 3).size == 2 * 4 * bb
        ks = tp.k_shard(w, qt, 4, 1024, 256, 768).reshape(4, 2 * bb)
        assert np.array_equal(ks, w.reshape(4, 4 * bb)[:, bb:3 * bb])
