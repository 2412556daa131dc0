"""acefa_flash_attn_ext_gen on the GPU: the mask given by its rule (causal,
sliding window, padding -- the masks acestep.cpp fills on the host,
src/qwen3-lm.h:597-609 and :872-881, src/dit-sampler.h:262-311) must give
exactly the output of acefa_flash_attn_ext with the equivalent 0 / -inf f16
mask: every tile class, visibility bit and added 0 is the same, so the
comparison is bit for bit.  The rule path launches no classification pass."""
import pytest
import torch

import acefa
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu


def _pair(c, mg, ne0=None, **kw):
    """(rule call, explicit-mask call, explicit-mask launch count)."""
    m = acefa.rule_mask(mg, c.B, c.n_q, c.n_kv, ne0=ne0)
    want = acefa.Op(c.q, c.k, c.v, mask=m, sinks=c.sinks, kv_type=c.kv_type, **kw)()
    torch.cuda.synchronize()
    n_explicit = acefa.last_launch_count()
    got = acefa.Op(c.q, c.k, c.v, sinks=c.sinks, kv_type=c.kv_type, mask_gen=mg, **kw)()
    torch.cuda.synchronize()
    assert acefa.device_error() == 0
    return got, want, n_explicit


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
def test_decode_causal_matches_validity_mask(kv):
    # batched CFG decode (qwen3-lm.h:872-881): set b sees keys 0 .. kv_pos[b]
    pos = [0, 350, 699, 511]
    c = Case(91, B=4, Hq=32, Hkv=8, n_q=1, n_kv=704, kv=kv, mask=None)
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=pos)
    got, want, _ = _pair(c, mg)
    assert torch.equal(got, want), float((got - want).abs().max())


def test_decode_split_kv_causal_and_padding():
    # 6000 keys: units split over CTAs, dead tail tiles skipped by the rule
    c = Case(92, B=2, Hq=16, Hkv=8, n_q=1, n_kv=6000, mask=None)
    for mg in (acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[4321, 63]),
               acefa.mask_gen(acefa.MASK_PADDING, lens=[6000, 1])):
        got, want, _ = _pair(c, mg)
        assert torch.equal(got, want), (mg.kind, float((got - want).abs().max()))


def test_decode_short_query_window():
    # FSQ-encoder-like node (S = 6 queries on the decode path) under a window
    c = Case(93, B=2, Hq=16, Hkv=16, n_q=6, n_kv=6, mask=None, sinks=True)
    got, want, _ = _pair(c, acefa.mask_gen(acefa.MASK_WINDOW, window=2))
    assert torch.equal(got, want)


def test_dense_prefill_causal_with_cache():
    # prefill of 300 tokens after 100 cached (qwen3-lm.h:597-609), padded window
    c = Case(94, B=1, Hq=16, Hkv=8, n_q=300, n_kv=512, mask=None)
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[100])
    got, want, n_explicit = _pair(c, mg)
    assert acefa.last_launch_count() == 1 and n_explicit == 2  # no classification pass
    assert torch.equal(got, want), float((got - want).abs().max())
    # and it is the operator: the oracle on the equivalent mask
    c.mask_cpu = acefa.rule_mask(mg, 1, 300, 512, device="cpu")
    assert_close(got.cpu().numpy(), c.oracle(), what="causal rule vs oracle")


@pytest.mark.parametrize("window", [0, 64, 200])
def test_dense_dit_window(window):
    # DiT sliding-window self-attention (dit-sampler.h:262-289), CFG batch of 2
    c = Case(95, B=2, Hq=16, Hkv=16, n_q=600, n_kv=600, mask=None)
    got, want, _ = _pair(c, acefa.mask_gen(acefa.MASK_WINDOW, window=window))
    assert torch.equal(got, want), float((got - want).abs().max())


def test_dense_cross_padding():
    # DiT cross-attention over padded encoder states (dit-sampler.h:291-311)
    c = Case(96, B=2, Hq=16, Hkv=8, n_q=500, n_kv=300, mask=None)
    got, want, _ = _pair(c, acefa.mask_gen(acefa.MASK_PADDING, lens=[200, 300]))
    assert torch.equal(got, want), float((got - want).abs().max())


def test_dense_rule_general_path_softcap_alibi():
    # softcap sends every tile down the general path; ALiBi slopes times the
    # rule's 0 add nothing, as they do for a 0 mask entry
    c = Case(97, B=1, Hq=8, Hkv=4, n_q=257, n_kv=390, mask=None)
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[133])
    got, want, _ = _pair(c, mg, softcap=30.0, max_bias=8.0)
    assert torch.equal(got, want), float((got - want).abs().max())


def test_rule_with_empty_rows_matches_mask():
    # padding length 0: every key hidden for batch 1 (the mask path's output too)
    c = Case(98, B=2, Hq=8, Hkv=8, n_q=200, n_kv=256, mask=None)
    got, want, _ = _pair(c, acefa.mask_gen(acefa.MASK_PADDING, lens=[256, 0]))
    assert torch.equal(got[0], want[0])
    assert torch.equal(torch.isnan(got[1]), torch.isnan(want[1]))
    assert torch.equal(torch.nan_to_num(got[1]), torch.nan_to_num(want[1]))


def test_rule_refusals():
    c = Case(99, B=2, Hq=8, Hkv=8, n_q=1, n_kv=64, mask=None)
    for mg in (acefa.mask_gen(0), acefa.mask_gen(acefa.MASK_WINDOW, window=-1)):
        with pytest.raises(acefa.AcefaError) as e:
            acefa.Op(c.q, c.k, c.v, mask_gen=mg)()
        assert e.value.status == -3  # ACEFA_ERR_SHAPE


@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
def test_dense_rules_over_bf16_and_q8_0(kv):
    """The rules on the dense path with converted K/V: the config-5 prompt
    prefill over a Q8_0 cache (causal) and a BF16 DiT window / padding node."""
    c = Case(97, B=1, Hq=32, Hkv=8, n_q=300, n_kv=512, kv=kv, max_seq=1024, s0=1, mask=None)
    got, want, _ = _pair(c, acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[100]))
    assert acefa.last_path() == 2
    assert torch.equal(got, want), float((got - want).abs().max())
    c2 = Case(98, B=2, Hq=16, Hkv=8, n_q=400, n_kv=400, kv=kv, mask=None)
    got, want, _ = _pair(c2, acefa.mask_gen(acefa.MASK_WINDOW, window=96))
    assert torch.equal(got, want), float((got - want).abs().max())
    got, want, _ = _pair(c2, acefa.mask_gen(acefa.MASK_PADDING, lens=[150, 400]))
    assert torch.equal(got, want), float((got - want).abs().max())
