#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own CPU contract — src/reference/*.cpp of
Frostbite1536/P100 compiled unmodified into oracle/_ref/ by oracle/Makefile —
and records its outputs:

* qmv-numerics.txt  the reference's tests/qmv_numerics.cpp table
                    (oracle/_ref/qmv_numerics), the golden file the reference
                    commits as docs/research/qmv-numerics-2026-10-10.txt;
* q8_1.npz          prepare() records (qd, qsum, q) for seeded activations with
                    edge cases: an all-zero block, outlier channels, large and
                    tiny magnitudes, exact .5 ties of x/d;
* qmv.npz           evaluate() results (q81, exact, weight_norm) for random_row
                    weights of every format at k = 256, 4096 and 14336;
* attention.npz     attention_reference() O and LSE for decode shapes (GQA 4:1
                    and 8:1, d = 64/128, seq_kv 1..450, a mask with a fully
                    masked case, softcap), and attention_tiled_model() with
                    split-K parts for one of them.

The reference is not present on the GPU box; the tests read only these files.
Usage: python tests/golden/make_golden.py   (needs oracle/_ref built)
"""
from __future__ import annotations

import pathlib
import subprocess
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent


def q8_1_cases(ref):
    rng = np.random.default_rng(20261201)
    rows = []
    x = rng.standard_normal(4096).astype(np.float32)
    x[:32] = 0                       # s = 0 block
    x[33] *= 50                      # outlier inside a block
    rows.append(x)
    rows.append((rng.standard_normal(4096) * 1000).astype(np.float32))     # large
    rows.append((rng.standard_normal(4096) * 1e-6).astype(np.float32))     # tiny: fp16 subnormal d
    y = rng.standard_normal(4096).astype(np.float32)
    y *= rng.standard_normal(4096).astype(np.float32) * 3                  # swiglu-like
    rows.append(y)
    # exact ties: per block amax = 127, so d = 1 and x/d = v; v = k + 0.5
    t = (rng.integers(-126, 126, 4096) + 0.5).astype(np.float32)
    t[::32] = 127.0
    rows.append(t)
    x = np.stack(rows)
    acts = np.stack([ref.prepare(r) for r in x])
    return dict(x=x, qd=acts["qd"], qsum=acts["qsum"], q=acts["q"].astype(np.int8))


def qmv_cases(ref):
    out = {}
    rng = np.random.default_rng(7)
    for t, name in oracle.TYPE_NAMES.items():
        for k in (256, 4096, 14336):
            rows = 17 if k < 14336 else 5
            w = ref.random_rows(t, k, rows, 60060 + k + t)
            x = rng.standard_normal((2, k)).astype(np.float32)
            x[0, :32] = 0
            x[1, 40] *= 50
            q81 = np.zeros((2, rows), np.float32)
            exact = np.zeros((2, rows), np.float64)
            wn = np.zeros(rows, np.float64)
            rb = w.size // rows
            for c in range(2):
                acts = ref.prepare(x[c])
                for r in range(rows):
                    e = ref.evaluate(t, w[r * rb:(r + 1) * rb], x[c], acts)
                    q81[c, r], exact[c, r], wn[r] = e["q81"], e["exact"], e["weight_norm"]
            key = f"{name}_{k}"
            out[key + "_w"] = w
            out[key + "_x"] = x
            out[key + "_q81"] = q81
            out[key + "_exact"] = exact
            out[key + "_wnorm"] = wn
    return out


ATTN_CASES = [
    # name, batch, hq, hkv, seq_kv, d, scale, softcap, mask
    ("gqa4_d128_s1", 1, 8, 2, 1, 128, 0.0, 0.0, None),
    ("gqa4_d128_s63", 1, 8, 2, 63, 128, 0.0, 0.0, None),
    ("gqa4_d128_s65", 1, 8, 2, 65, 128, 0.0, 0.0, None),
    ("gqa4_d128_s450", 2, 4, 1, 450, 128, 0.0, 0.0, None),
    ("gqa8_d128_s300", 1, 8, 1, 300, 128, 0.0, 0.0, None),
    ("gqa1_d64_s257", 1, 4, 4, 257, 64, 0.0, 0.0, None),
    ("softcap_d128_s129", 1, 4, 1, 129, 128, 0.5, 30.0, None),
    ("masked_d128_s200", 1, 4, 1, 200, 128, 0.0, 0.0, "partial"),
    ("allmasked_d128_s70", 1, 4, 1, 70, 128, 0.0, 0.0, "all"),
]


def attention_cases(ref):
    out = {}
    rng = np.random.default_rng(12345)
    for name, b, hq, hkv, s, d, scale, softcap, mask_kind in ATTN_CASES:
        p = oracle.Attn(batch=b, n_head_q=hq, n_head_kv=hkv, seq_q=1, seq_kv=s, d_qk=d, d_v=d, scale=scale,
                        softcap=softcap)
        qs, ks, vs, _, _ = p.shapes()
        q = rng.standard_normal(qs).astype(np.float32)
        k = (rng.standard_normal(ks) * 0.5).astype(np.float16)
        v = (rng.standard_normal(vs) * 0.5).astype(np.float16)
        mask = None
        if mask_kind == "partial":
            mask = np.where(rng.random((1, s)) < 0.3, -np.inf, rng.standard_normal((1, s)) * 0.1).astype(np.float32)
        elif mask_kind == "all":
            mask = np.full((1, s), -np.inf, np.float32)
        o, lse = ref.attention_reference(p, q, k.astype(np.float32), v.astype(np.float32), mask)
        out[name + "_q"] = q
        out[name + "_k"] = k
        out[name + "_v"] = v
        if mask is not None:
            out[name + "_mask"] = mask
        out[name + "_o"] = o
        out[name + "_lse"] = lse
        out[name + "_params"] = np.array([b, hq, hkv, s, d], np.int32)
        out[name + "_scales"] = np.array([scale, softcap], np.float32)
    # Split-K model (FP32 P and O, four parts) for one case.
    name = "gqa4_d128_s450"
    b, hq, hkv, s, d = out[name + "_params"]
    p = oracle.Attn(batch=int(b), n_head_q=int(hq), n_head_kv=int(hkv), seq_q=1, seq_kv=int(s), d_qk=int(d),
                    d_v=int(d))
    cfg = oracle.Tiled(1, 64, False, False, False, kv_parallel_blocks=4)
    o, lse = ref.attention_tiled(p, cfg, out[name + "_q"], out[name + "_k"].astype(np.float32),
                                 out[name + "_v"].astype(np.float32))
    out[name + "_split4_o"] = o
    out[name + "_split4_lse"] = lse
    return out


def main():
    if not oracle.Ref.available():
        sys.exit("oracle/_ref is not built: run make -C oracle with the reference sources present")
    ref = oracle.Ref()
    table = subprocess.run([str(ROOT / "oracle" / "_ref" / "qmv_numerics")], check=True, capture_output=True,
                           text=True).stdout
    (OUT / "qmv-numerics.txt").write_text(table)
    np.savez_compressed(OUT / "q8_1.npz", **q8_1_cases(ref))
    np.savez_compressed(OUT / "qmv.npz", **qmv_cases(ref))
    np.savez_compressed(OUT / "attention.npz", **attention_cases(ref))
    for f in sorted(OUT.glob("*")):
        if f.suffix in (".npz", ".txt"):
            print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
