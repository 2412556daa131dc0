"""CPU: the mask rules of acefa_flash_attn_ext_gen stand for exactly the f16
masks acestep.cpp fills on the host.  acefa.rule_mask (the tensor a rule is
bit-identical to, used by the GPU tests) is checked element for element against
a restatement of the reference's fill loops:
  * LM prefill causal mask, src/qwen3-lm.h:597-609 (row i sees j <= kv_pos + i,
    padded tail -inf);
  * batched decode validity mask, src/qwen3-lm.h:872-881 (set b sees
    j < kv_pos[b] + 1);
  * DiT sliding window, src/dit-sampler.h:262-289 (|qi - ki| <= win, window
    off when win <= 0 or S <= win: then the node is unmasked);
  * DiT cross-attention padding, src/dit-sampler.h:291-311 (ki < real_enc_S[b])."""
import numpy as np
import pytest
import torch

import acefa

NEG = np.float16(-np.inf)


def _f16(x):
    return torch.from_numpy(np.asarray(x, dtype=np.float16))


def ref_causal(n_kv_pad, n_tokens, kv_pos):
    m = np.empty((n_tokens, n_kv_pad), np.float16)
    for i in range(n_tokens):
        for j in range(n_kv_pad):
            m[i, j] = 0.0 if j <= kv_pos + i else NEG
    return m


def ref_decode(n_kv_pad, kv_pos):
    m = np.empty((len(kv_pos), n_kv_pad), np.float16)
    for b, p in enumerate(kv_pos):
        kvl = p + 1
        for j in range(n_kv_pad):
            m[b, j] = 0.0 if j < kvl else NEG
    return m


def ref_window(S, win):
    m = np.empty((S, S), np.float16)
    for qi in range(S):
        for ki in range(S):
            dist = abs(qi - ki)
            m[qi, ki] = 0.0 if (win <= 0 or S <= win or dist <= win) else NEG
    return m


def ref_padding(S, enc_S, real):
    m = np.empty((len(real), S, enc_S), np.float16)
    for b, re in enumerate(real):
        for qi in range(S):
            for ki in range(enc_S):
                m[b, qi, ki] = 0.0 if ki < re else NEG
    return m


@pytest.mark.parametrize("kv_pos,n_tokens,n_kv_pad", [(0, 7, 256), (100, 33, 256), (200, 56, 256)])
def test_causal_rule_is_the_prefill_mask(kv_pos, n_tokens, n_kv_pad):
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[kv_pos])
    got = acefa.rule_mask(mg, 1, n_tokens, n_kv_pad, device="cpu")[0, 0]
    assert torch.equal(got.view(torch.int16), _f16(ref_causal(n_kv_pad, n_tokens, kv_pos)).view(torch.int16))


def test_causal_rule_is_the_decode_validity_mask():
    kv_pos = [0, 5, 255, 97, 128, 31]
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=kv_pos)
    got = acefa.rule_mask(mg, len(kv_pos), 1, 256, device="cpu")[:, 0, 0]
    assert torch.equal(got.view(torch.int16), _f16(ref_decode(256, kv_pos)).view(torch.int16))


@pytest.mark.parametrize("S,win", [(50, 8), (50, 1), (64, 63), (40, 0), (40, 40), (40, 100)])
def test_window_rule_is_sa_mask_sw(S, win):
    want = _f16(ref_window(S, win))
    if win <= 0 or S <= win:
        # the reference fills all zeros: the node runs unmasked (no rule, no mask)
        assert not torch.isinf(want.float()).any()
        return
    mg = acefa.mask_gen(acefa.MASK_WINDOW, window=win)
    got = acefa.rule_mask(mg, 2, S, S, device="cpu")
    for b in range(2):
        assert torch.equal(got[b, 0].view(torch.int16), want.view(torch.int16))


def test_padding_rule_is_ca_mask():
    real = [17, 64, 0, 40]
    mg = acefa.mask_gen(acefa.MASK_PADDING, lens=real)
    got = acefa.rule_mask(mg, len(real), 20, 64, device="cpu")[:, 0]
    assert torch.equal(got.view(torch.int16), _f16(ref_padding(20, 64, real)).view(torch.int16))
