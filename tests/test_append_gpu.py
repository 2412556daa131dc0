"""acefa_flash_attn_ext_append on the GPU: the decode op fused with the
KV-cache append that precedes it (ggml_set_rows of the new K and V rows,
src/qwen3-lm.h:776-777).  The fused call must leave exactly the cache a
separate append would (F16 / BF16 rounding, Q8_0 blocks bit-exact with ggml's
quantiser) and produce exactly the output of acefa_flash_attn_ext on that
cache: both kernels are deterministic, so the comparison is bit for bit."""
import pytest
import torch

import acefa
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu


def _convert(x, kv):
    if kv == "f16":
        return x.half()
    if kv == "bf16":
        return x.bfloat16()
    return acefa.quantize_q8_0(x)


def _run(kv, B, Hq, Hkv, n_kv, pos, max_seq=None, seed=81):
    """Fused call vs (append with torch, then the plain operator)."""
    valid = [p + 1 for p in pos]  # decode visibility: keys 0 .. kv_pos
    c = Case(seed, B=B, Hq=Hq, Hkv=Hkv, n_q=1, n_kv=n_kv, kv=kv, max_seq=max_seq, mask="valid", valid=valid)
    g = torch.Generator().manual_seed(seed + 1)
    k_new = torch.randn(B, Hkv, 1, 128, generator=g).cuda()
    v_new = torch.randn(B, Hkv, 1, 128, generator=g).cuda()
    pos_t = torch.tensor(pos, dtype=torch.int64, device="cuda")
    # reference: rows written by torch, then the existing entry point
    k_ref, v_ref = c.k_cache.clone(), c.v_cache.clone()
    for b, p in enumerate(pos):
        k_ref[b, :, p] = _convert(k_new[b, :, 0], kv)
        v_ref[b, :, p] = _convert(v_new[b, :, 0], kv)
    want = acefa.flash_attn_ext(c.q, k_ref[:, :, :n_kv], v_ref[:, :, :n_kv], c.mask, kv_type=c.kv_type)
    torch.cuda.synchronize()
    # fused: the same cache before the append
    op = acefa.Op(c.q, c.k, c.v, mask=c.mask, kv_type=c.kv_type, k_new=k_new, v_new=v_new, pos=pos_t)
    got = op()
    torch.cuda.synchronize()
    assert acefa.device_error() == 0
    assert torch.equal(c.k_cache.view(torch.uint8), k_ref.view(torch.uint8)), "K cache differs"
    assert torch.equal(c.v_cache.view(torch.uint8), v_ref.view(torch.uint8)), "V cache differs"
    assert torch.equal(got, want), float((got - want).abs().max())
    return c, got


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
def test_append_decode_matches_separate_append(kv):
    # config-2-like step: 4 sets at different positions, first/last/middle rows
    c, got = _run(kv, B=4, Hq=32, Hkv=8, n_kv=700, pos=[0, 350, 699, 511], max_seq=1024)
    if kv == "f16":
        # and the result is the operator's (within the usual tolerance of the oracle)
        c.k_cache_cpu = c.k_cache.cpu()
        c.v_cache_cpu = c.v_cache.cpu()
        assert_close(got.cpu().numpy(), c.oracle(), what="append f16 vs oracle")


def test_append_split_kv_units():
    # 6000 keys: each (set, head) unit is split over several CTAs; the row's tile
    # belongs to one of them, which writes it before reading that tile
    _run("f16", B=2, Hq=16, Hkv=8, n_kv=6000, pos=[4321, 64])


def test_append_position_out_of_range_reports_error():
    c = Case(82, B=2, Hq=16, Hkv=8, n_q=1, n_kv=300, mask="zeros")
    k_new = torch.randn(2, 8, 1, 128, device="cuda")
    v_new = torch.randn(2, 8, 1, 128, device="cuda")
    before = c.k_cache.clone()
    op = acefa.Op(c.q, c.k, c.v, mask=c.mask, k_new=k_new, v_new=v_new,
                  pos=torch.tensor([300, -1], dtype=torch.int64, device="cuda"))
    op()
    torch.cuda.synchronize()
    assert acefa.device_error() == 5  # DEVERR_APPEND_POS; the error word is cleared by the read
    assert torch.equal(c.k_cache, before)  # nothing written
    assert acefa.device_error() == 0


def test_append_refuses_dense_shapes():
    c = Case(83, B=1, Hq=16, Hkv=8, n_q=200, n_kv=300, mask=None)
    k_new = torch.randn(1, 8, 1, 128, device="cuda")
    with pytest.raises(acefa.AcefaError):
        acefa.Op(c.q, c.k, c.v, k_new=k_new, v_new=k_new.clone(),
                 pos=torch.zeros(1, dtype=torch.int64, device="cuda"))()


def test_append_q8_0_three_ctas_per_sm():
    """16 sets x 8 heads over 1536 keys: the Q8_0 instance with three CTAs per
    SM (decode_wide), new rows in different tiles and CTA ranges of each set."""
    pos = [100 + 89 * b for b in range(16)]
    _run("q8_0", B=16, Hq=32, Hkv=8, n_kv=1536, pos=pos, max_seq=2048, seed=83)
