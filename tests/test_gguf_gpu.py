"""A llama GGUF file loaded into the decoder (p100_b200.gguf.load_llama) on
B200.  The decoder's own random model is written out under llama.cpp's
tensor names (q, k, v and gate, up split back out of the fused matrices)
and read back into a second decoder: both must decode the same tokens with
the same logits, bit for bit, which checks every tensor's placement — also
for a file that mixes formats per matrix as llama.cpp's Q4_K_M files do."""
import numpy as np
import pytest

import p100_b200 as P
from p100_b200 import gguf

pytestmark = pytest.mark.gpu
TINY = dict(n_layer=2, hidden=256, n_head=4, n_head_kv=2, head_dim=64, ffn=512, vocab=300, max_ctx=512)


def export(dec, cfg):
    """The decoder's tensors as a llama GGUF tensor list (each matrix in its
    own format; the fused q|k|v and gate|up ranges split back out)."""
    types = cfg.types()
    H, hd, F, V = cfg.hidden, cfg.head_dim, cfg.ffn, cfg.vocab
    nq, nkv = cfg.n_head, cfg.n_head_kv

    def t(which, layer=0):
        ptr, nbytes, _, _ = dec.tensor(which, layer)
        return dec.read(ptr, nbytes)
    gt = lambda i: gguf.GGML_OF_P100[types[i]]
    lt = lambda l, part: types[P.tt_layer(l, part)]
    nbytes = lambda qt, rows, k: rows * (k // P.BLOCK_ELEMS[qt] * P.BLOCK_BYTES[qt])
    out = [("token_embd.weight", gt(P.TT_EMBED), (H, V), t(P.T_EMBED)),
           ("output_norm.weight", gguf.GGML_F32, (H,), t(P.T_OUT_NORM)),
           ("output.weight", gt(P.TT_LM_HEAD), (H, V), t(P.T_LM_HEAD))]
    for l in range(cfg.n_layer):
        b = f"blk.{l}."
        qkv = t(P.T_WQKV, l)
        gu = t(P.T_WGATE_UP, l)
        qn, kn = nbytes(lt(l, P.TT_Q), nq * hd, H), nbytes(lt(l, P.TT_K), nkv * hd, H)
        gn = nbytes(lt(l, P.TT_GATE), F, H)
        assert qkv.size == qn + kn + nbytes(lt(l, P.TT_V), nkv * hd, H)
        assert gu.size == gn + nbytes(lt(l, P.TT_UP), F, H)
        g = lambda part: gguf.GGML_OF_P100[lt(l, part)]
        out += [(b + "attn_norm.weight", gguf.GGML_F32, (H,), t(P.T_ATTN_NORM, l)),
                (b + "attn_q.weight", g(P.TT_Q), (H, nq * hd), qkv[:qn]),
                (b + "attn_k.weight", g(P.TT_K), (H, nkv * hd), qkv[qn:qn + kn]),
                (b + "attn_v.weight", g(P.TT_V), (H, nkv * hd), qkv[qn + kn:]),
                (b + "attn_output.weight", g(P.TT_O), (nq * hd, H), t(P.T_WO, l)),
                (b + "ffn_norm.weight", gguf.GGML_F32, (H,), t(P.T_FFN_NORM, l)),
                (b + "ffn_gate.weight", g(P.TT_GATE), (H, F), gu[:gn]),
                (b + "ffn_up.weight", g(P.TT_UP), (H, F), gu[gn:]),
                (b + "ffn_down.weight", g(P.TT_DOWN), (F, H), t(P.T_WDOWN, l))]
    meta = {"general.architecture": "llama", "llama.block_count": cfg.n_layer, "llama.embedding_length": H,
            "llama.attention.head_count": nq, "llama.attention.head_count_kv": nkv, "llama.feed_forward_length": F,
            "llama.context_length": cfg.max_ctx, "llama.rope.freq_base": cfg.rope_theta,
            "llama.attention.layer_norm_rms_epsilon": cfg.norm_eps, "llama.rope.dimension_count": hd}
    return meta, out


def run(dec, steps):
    dec.fill_kv(100, 3, 0.5)
    dec.set_state(100, 7)
    toks, logits = [], []
    for _ in range(steps):
        dec.step(1)
        toks.append(dec.state()[1])
        logits.append(dec.read(*dec.buffer(P.B_LOGITS)).copy())
    return toks, logits


def q4_k_m_types(n_layer):
    """llama.cpp Q4_K_M-like formats: Q4_K, with attn_v and ffn_down in Q6_K
    in alternate layers, the output matrix in Q6_K, one ffn_up in Q5_K and
    one attn_k in Q8_0 (a fused q|k|v of three formats)."""
    t = [P.Q4_K] * P.dec_tensor_types(n_layer)
    t[P.TT_LM_HEAD] = P.Q6_K
    for l in range(0, n_layer, 2):
        t[P.tt_layer(l, P.TT_V)] = P.Q6_K
        t[P.tt_layer(l, P.TT_DOWN)] = P.Q6_K
    t[P.tt_layer(n_layer - 1, P.TT_UP)] = P.Q5_K
    t[P.tt_layer(n_layer - 1, P.TT_K)] = P.Q8_0
    return t


MIXED = -1


@pytest.mark.parametrize("wtype", [P.Q4_0, P.Q8_0, P.Q4_K, MIXED], ids=["q4_0", "q8_0", "q4_k", "q4_k_m"])
@pytest.mark.parametrize("kv_type", [P.KV_F16, P.KV_Q8_0])
def test_decoder_round_trips_through_gguf(cuda, tmp_path, wtype, kv_type):
    types = None
    if wtype == MIXED:
        wtype, types = P.Q4_K, q4_k_m_types(TINY["n_layer"])
    cfg = P.LlamaConfig(**TINY, wtype=wtype, kv_type=kv_type, tensor_types=types)
    dec = P.Decoder(cfg)
    try:
        dec.init_random(2024 + wtype)
        meta, tensors = export(dec, cfg)
        toks, logits = run(dec, 3)
    finally:
        dec.close()
    path = tmp_path / "model.gguf"
    gguf.write_gguf(path, meta, tensors)
    dec2 = gguf.load_llama(str(path), max_ctx=cfg.max_ctx, kv_type=kv_type)
    try:
        assert dec2.cfg.wtype == wtype and dec2.cfg.vocab == cfg.vocab and dec2.cfg.types() == cfg.types()
        toks2, logits2 = run(dec2, 3)
    finally:
        dec2.close()
    assert toks2 == toks
    for a, b in zip(logits, logits2):
        assert np.array_equal(a, b)
