"""CPU tests of the oracle: Q8_0 pinned against gguf, attention cross-checked
against independent float64 fixtures, the ggml-cpu (F16 accumulation)
mode's known drift, and the QK-norm + RoPE prologue pinned against the Qwen3
model definition."""
import glob
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_matches_gguf_bit_exact(oracle_mod):
    x = np.load(os.path.join(GOLDEN, "q8_0_input.npy"))
    want = np.load(os.path.join(GOLDEN, "q8_0_gguf.npy"))
    got = oracle_mod.quantize_q8_0(x)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_q8_0_dequant_roundtrip(oracle_mod):
    x = np.load(os.path.join(GOLDEN, "q8_0_input.npy"))
    y = oracle_mod.quantize_q8_0(x)
    xr = oracle_mod.dequantize_q8_0(y)
    blocks = x.reshape(x.shape[0], -1, 32)
    d = np.abs(blocks).max(-1, keepdims=True) / np.float32(127.0)
    d16 = d.astype(np.float16).astype(np.float32)
    err = np.abs(xr.reshape(blocks.shape) - blocks)
    # half a quantisation step plus the f16 rounding of the block scale
    assert np.all(err <= 0.5 * d * (1 + 1e-5) + 127.0 * np.abs(d - d16) + 1e-30)


def _load_case(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_case_*.npz"))),
                         ids=lambda p: os.path.basename(p)[10:-4])
def test_oracle_matches_float64_fixtures(oracle_mod, path):
    c = _load_case(path)
    out = oracle_mod.flash_attn_ext(c["q"], c["k"], c["v"], c.get("mask"), c.get("sinks"), scale=float(c["scale"]),
                                    max_bias=float(c["max_bias"]), softcap=float(c["softcap"]))
    np.testing.assert_allclose(out, c["out"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_case_*.npz"))),
                         ids=lambda p: os.path.basename(p)[10:-4])
def test_ggml_cpu_mode_close_to_f32(oracle_mod, path):
    """The ggml-cpu restatement (F16 Q and V accumulator) drifts but stays close."""
    c = _load_case(path)
    kw = dict(scale=float(c["scale"]), max_bias=float(c["max_bias"]), softcap=float(c["softcap"]))
    ref = oracle_mod.flash_attn_ext(c["q"], c["k"], c["v"], c.get("mask"), c.get("sinks"), **kw)
    g = oracle_mod.flash_attn_ext(c["q"], c["k"], c["v"], c.get("mask"), c.get("sinks"),
                                  mode=oracle_mod.MODE_GGML_CPU, **kw)
    assert np.abs(g - ref).max() < 2e-2
    # rows with no visible key are exactly zero in both modes
    assert np.array_equal(ref == 0, g == 0) or np.abs(g - ref).max() < 2e-2


def test_all_masked_row_is_zero(oracle_mod):
    rng = np.random.default_rng(42)
    q = rng.standard_normal((1, 2, 3, 64)).astype(np.float32)
    k = rng.standard_normal((1, 1, 10, 64)).astype(np.float16)
    v = rng.standard_normal((1, 1, 10, 64)).astype(np.float16)
    m = np.zeros((1, 1, 3, 10), np.float16)
    m[0, 0, 1, :] = -np.inf
    out = oracle_mod.flash_attn_ext(q, k, v, m, scale=0.125)
    assert np.all(out[0, 1] == 0.0)
    assert np.all(np.abs(out[0, 0]) > 0)


def test_q8_0_kv_oracle_equals_dequantised_f32(oracle_mod):
    rng = np.random.default_rng(43)
    q = rng.standard_normal((2, 4, 1, 128)).astype(np.float32)
    kf = rng.standard_normal((2, 2, 70, 128)).astype(np.float32)
    vf = rng.standard_normal((2, 2, 70, 128)).astype(np.float32)
    kq, vq = oracle_mod.quantize_q8_0(kf), oracle_mod.quantize_q8_0(vf)
    a = oracle_mod.flash_attn_ext(q, kq, vq, scale=0.088, k_type=oracle_mod.GGML_Q8_0, v_type=oracle_mod.GGML_Q8_0)
    b = oracle_mod.flash_attn_ext(q, oracle_mod.dequantize_q8_0(kq), oracle_mod.dequantize_q8_0(vq), scale=0.088)
    np.testing.assert_allclose(a, b, atol=1e-6, rtol=1e-6)


def test_contract_violations_rejected(oracle_mod):
    q = np.zeros((1, 3, 1, 64), np.float32)  # Hq = 3
    k = np.zeros((1, 2, 8, 64), np.float16)  # Hkv = 2 does not divide 3
    with pytest.raises(ValueError):
        oracle_mod.flash_attn_ext(q, k, k, scale=1.0)


@pytest.mark.parametrize("name", ["d128", "d64"])
def test_rope_norm_matches_qwen3_definition(oracle_mod, name):
    """QK-norm + RoPE NEOX against HF transformers' Qwen3 modules
    (tests/golden/make_rope_golden.py).  RMSNorm agrees to f32 rounding; the
    rotation to f32 rounding of the angle pos * inv_freq (the two sides compute
    inv_freq by different f32 expressions, so the angle may differ by ~pos * 1e-7
    rad): the bound per row is 2e-6 + 1.2e-7 * pos * max|x|."""
    z = np.load(os.path.join(GOLDEN, f"rope_norm_{name}.npz"))
    normed = oracle_mod.rope_norm(z["x"], z["weight"], float(z["eps"]), 0.0, None)
    np.testing.assert_allclose(normed, z["normed"], rtol=2e-6, atol=2e-6)
    out = oracle_mod.rope_norm(z["x"], z["weight"], float(z["eps"]), float(z["theta"]), z["positions"])
    err = np.abs(out - z["out"]).max(axis=1)
    bound = 2e-6 + 1.2e-7 * z["positions"].astype(np.float64) * np.abs(z["normed"]).max(axis=1)
    assert (err <= bound).all(), (err, bound)
    # without a weight nothing is normalised; without theta nothing rotates
    x = z["x"][:2]
    assert np.array_equal(oracle_mod.rope_norm(x, None, 1e-6, 0.0, None), x)


@pytest.mark.parametrize("B,Hq,Hkv,nq,nkv,kind", [(2, 8, 2, 1, 300, "valid"), (1, 8, 4, 40, 70, "causal"),
                                                  (2, 4, 4, 33, 33, "window"), (1, 6, 2, 17, 45, "holes")])
def test_oracle_matches_torch_sdpa(oracle_mod, B, Hq, Hkv, nq, nkv, kind):
    """The oracle's F32 mode against an implementation it shares no code with:
    PyTorch's scaled_dot_product_attention in float64 on the CPU (GQA by head
    repetition), for the parts of the contract SDPA expresses -- scale, GQA,
    additive 0 / -inf masks in the shapes acestep.cpp builds.  Rows with no
    visible key are left out (SDPA returns NaN there, ggml 0)."""
    import torch

    rng = np.random.default_rng(77 + nq)
    D = 64
    q = rng.standard_normal((B, Hq, nq, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, nkv, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, nkv, D)).astype(np.float16)
    i = np.arange(nq)[:, None]
    j = np.arange(nkv)[None, :]
    if kind == "valid":
        vis = np.stack([j < 150, j < 300])[:, None].repeat(nq, axis=1)[:, :, 0][:, None]
        vis = np.broadcast_to(vis, (B, 1, nq, nkv))
    elif kind == "causal":
        vis = np.broadcast_to(j <= i + (nkv - nq), (B, 1, nq, nkv))
    elif kind == "window":
        vis = np.broadcast_to(np.abs(i - j) <= 5, (B, 1, nq, nkv))
    else:
        vis = np.broadcast_to(rng.random((1, 1, nq, nkv)) < 0.6, (B, 1, nq, nkv))
    mask = np.where(vis, 0.0, -np.inf).astype(np.float16)
    scale = D ** -0.5
    got = oracle_mod.flash_attn_ext(q, k, v, mask, None, scale=scale)  # (B, nq, Hq, D)
    rep = Hq // Hkv
    tq = torch.from_numpy(q).double()
    tk = torch.from_numpy(k.astype(np.float32)).double().repeat_interleave(rep, dim=1)
    tv = torch.from_numpy(v.astype(np.float32)).double().repeat_interleave(rep, dim=1)
    tm = torch.from_numpy(mask.astype(np.float32)).double()
    want = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv, attn_mask=tm, scale=scale)
    want = want.permute(0, 2, 1, 3).numpy()  # (B, nq, Hq, D)
    rows = vis[:, 0].any(axis=-1)  # (B, nq)
    sel = np.broadcast_to(rows[:, :, None, None], want.shape)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got[sel], want[sel], rtol=0, atol=2e-5)


def _reference_cfg_loop(batch_logits, n_active, out_V, eos_idx, code_offset, code_count, cfg_scale, use_cfg):
    """The host loop of src/pipeline-lm.cpp:471-492 restated with numpy f32
    scalars (each operation rounded to f32, as the reference's C++ computes
    it): combine in place on the EOS column and the code range, then copy the
    compact array of each active sequence."""
    lg = batch_logits.copy()
    s = np.float32(cfg_scale)
    out = np.empty((n_active, code_count + 1), dtype=np.float32)
    for a in range(n_active):
        lc = lg[a * out_V:(a + 1) * out_V]
        if use_cfg:
            lu = lg[(n_active + a) * out_V:(n_active + a + 1) * out_V]
            lc[eos_idx] = lu[eos_idx] + s * (lc[eos_idx] - lu[eos_idx])
            for c in range(code_count):
                i = code_offset + c
                lc[i] = lu[i] + s * (lc[i] - lu[i])
        out[a, 0] = lc[eos_idx]
        out[a, 1:] = lc[code_offset:code_offset + code_count]
    return out


@pytest.mark.parametrize("use_cfg", [True, False])
def test_cfg_logit_combine_matches_reference_loop(oracle_mod, use_cfg):
    """Small partial-head layout (EOS at column 0, codes from column 24 as with
    lm_offset = TOKEN_IM_END) with extreme values in the mix."""
    n, V, eos, off, cnt = 3, 97, 0, 24, 70
    r = np.random.default_rng(11)
    logits = (r.standard_normal(2 * n * V) * 30).astype(np.float32)
    logits[[5, 40, 300, 400]] = [np.inf, -np.inf, 3.0e38, -1.0e9]
    want = _reference_cfg_loop(logits, n, V, eos, off, cnt, 3.5, use_cfg)
    rows = logits.reshape(2 * n, V)
    got = oracle_mod.cfg_logit_combine(rows[:n], rows[n:] if use_cfg else None, eos, off, cnt, 3.5)
    assert np.array_equal(got, want, equal_nan=True)
