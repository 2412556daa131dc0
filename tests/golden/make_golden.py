"""Regenerate the committed fixtures in tests/golden/.

    python tests/golden/make_golden.py

1. q8_0_input.npy / q8_0_gguf.npy -- seeded rows (including ties, zeros and
   extreme magnitudes) quantised by the gguf 0.19.0 package's Q8_0
   implementation, which states bit-exactness with ggml-quants.c.  These pin the
   Q8_0 block format used by the oracle, the torch quantiser and the kernels.
2. attn_case_*.npz -- small ggml_flash_attn_ext cases (GQA, strided masks with
   -inf, head/batch broadcast, ALiBi, softcap, sinks, all-masked rows) evaluated
   by an independent float64 numpy statement of the operator written in this
   file.  They cross-check the C oracle; they are not reference outputs (the
   reference's ggml kernels are not in its tree).

Seeds: base 42, the reference's own test seed (tests/debug-dit-cossim.py:17).
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_0_fixture():
    import gguf

    rng = np.random.default_rng(42)
    rows = [rng.standard_normal(256).astype(np.float32) for _ in range(6)]
    rows.append(np.zeros(256, np.float32))
    r = rng.standard_normal(256).astype(np.float32)
    r[:32] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32) / 127.0 * 2.0  # exact .5 ties
    rows.append(r)
    rows.append((rng.standard_normal(256) * 1e4).astype(np.float32))
    rows.append((rng.standard_normal(256) * 1e-6).astype(np.float32))
    x = np.stack(rows)
    y = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    np.save(os.path.join(HERE, "q8_0_input.npy"), x)
    np.save(os.path.join(HERE, "q8_0_gguf.npy"), np.asarray(y, dtype=np.uint8))


def ref_attention_f64(q, k, v, mask, sinks, scale, max_bias, softcap):
    """float64 ggml_flash_attn_ext: q (B,Hq,nq,D) k/v (Bk,Hkv,nkv,D) mask (Bm,Hm,>=nq,>=nkv)."""
    B, Hq, nq, D = q.shape
    Bk, Hkv, nkv, Dv = v.shape
    out = np.zeros((B, nq, Hq, Dv), np.float64)
    nhl2 = 1 << int(np.floor(np.log2(Hq)))
    m0 = 2.0 ** (-max_bias / nhl2)
    m1 = 2.0 ** (-(max_bias / 2.0) / nhl2)
    for b in range(B):
        for h in range(Hq):
            slope = 1.0 if max_bias <= 0 else (m0 ** (h + 1) if h < nhl2 else m1 ** (2 * (h - nhl2) + 1))
            kk = k[b // (B // Bk), h // (Hq // Hkv)].astype(np.float64)
            vv = v[b // (B // Bk), h // (Hq // Hkv)].astype(np.float64)
            s = q[b, h].astype(np.float64) @ kk.T
            if softcap:
                s = softcap * np.tanh(s * (scale / softcap))
            else:
                s = s * scale
            if mask is not None:
                mm = mask[b % mask.shape[0], h % mask.shape[1], :nq, :nkv].astype(np.float64)
                s = s + slope * mm
            logits = s
            if sinks is not None:
                logits = np.concatenate([s, np.full((nq, 1), float(sinks[h]))], axis=1)
            mx = np.max(logits, axis=1, keepdims=True)
            valid = np.isfinite(mx)
            mxs = np.where(valid, mx, 0.0)
            p = np.exp(logits - mxs)
            den = p.sum(axis=1, keepdims=True)
            o = p[:, :nkv] @ vv
            o = np.where(den > 0, o / np.where(den > 0, den, 1.0), 0.0)
            out[b, :, h, :] = o
    return out.astype(np.float32)


def attn_fixtures():
    rng = np.random.default_rng(42 + 1000 * 9)
    cases = []
    # (name, B, Bk, Hq, Hkv, nq, nkv, D, mask kind, Hm, Bm, max_bias, softcap, sinks)
    specs = [
        ("decode_gqa2", 1, 1, 4, 2, 1, 100, 64, "tail", 1, 1, 0.0, 0.0, False),
        ("decode_batch_cfg", 4, 4, 8, 2, 1, 130, 64, "tail", 1, 4, 0.0, 0.0, False),
        ("prefill_causal", 1, 1, 2, 1, 20, 20, 64, "causal", 1, 1, 0.0, 0.0, False),
        ("window_bidir", 2, 2, 4, 4, 24, 24, 64, "window", 1, 2, 0.0, 0.0, False),
        ("cross_padding", 2, 2, 2, 2, 9, 33, 64, "padding", 1, 2, 0.0, 0.0, False),
        ("alibi_softcap", 1, 1, 6, 3, 3, 40, 64, "random", 1, 1, 8.0, 30.0, False),
        ("sinks_allmasked", 2, 1, 4, 2, 4, 17, 64, "rowdead", 2, 1, 0.0, 0.0, True),
        ("nomask_kvbroadcast", 2, 1, 2, 1, 3, 50, 128, None, 1, 1, 0.0, 0.0, False),
    ]
    for (name, B, Bk, Hq, Hkv, nq, nkv, D, mk, Hm, Bm, mb, sc, sk) in specs:
        q = rng.standard_normal((B, Hq, nq, D)).astype(np.float32)
        k = rng.standard_normal((Bk, Hkv, nkv, D)).astype(np.float16)
        v = rng.standard_normal((Bk, Hkv, nkv, D)).astype(np.float16)
        mask = None
        if mk is not None:
            npad = nkv + 3  # mask rows wider than n_kv, like acestep's padded windows
            mask = np.zeros((Bm, Hm, nq + 2, npad), np.float16)
            for b in range(Bm):
                for h in range(Hm):
                    for i in range(nq + 2):
                        for j in range(npad):
                            if mk == "tail":
                                ok = j < nkv - 7 * b - 1
                            elif mk == "causal":
                                ok = j <= i
                            elif mk == "window":
                                ok = abs(i - j) <= 5
                            elif mk == "padding":
                                ok = j < nkv - 4 - b
                            elif mk == "random":
                                ok = rng.random() < 0.7
                            elif mk == "rowdead":
                                ok = (i % 2 == 0) and j < nkv - 2
                            mask[b, h, i, j] = 0.0 if ok else -np.inf
            if mk == "random":
                mask[mask == 0] = (rng.standard_normal(int((mask == 0).sum())) * 0.5).astype(np.float16)
        sinks = rng.standard_normal(Hq).astype(np.float32) if sk else None
        scale = 1.0 / np.sqrt(D)
        out = ref_attention_f64(q, k, v, mask, sinks, scale, mb, sc)
        arrays = dict(q=q, k=k, v=v, out=out, scale=np.float32(scale), max_bias=np.float32(mb),
                      softcap=np.float32(sc))
        if mask is not None:
            arrays["mask"] = mask
        if sinks is not None:
            arrays["sinks"] = sinks
        np.savez_compressed(os.path.join(HERE, f"attn_case_{name}.npz"), **arrays)
        cases.append(name)
    return cases


if __name__ == "__main__":
    q8_0_fixture()
    print("cases:", attn_fixtures())
