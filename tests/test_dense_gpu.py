"""GPU parity of the dense tcgen05 path (LM prefill, encoders, DiT self/cross)
against the CPU oracle, through the C ABI.  Same tolerance as the decode path:
max-abs 2e-3, cosine >= 0.99995 vs the FP32 oracle; mask indexing bit-exact."""
import numpy as np
import pytest
import torch

import acefa
import oracle
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu


def run_case(case, rows=None, **kw):
    got = case.gpu(**kw)
    assert acefa.last_path() == 2, "expected the dense tcgen05 path"
    if rows is None:
        want = case.oracle(**kw)
    else:
        want = oracle_rows(case, rows, **kw)
        got = got[:, rows]
    assert_close(got, want, what=str(kw))
    assert acefa.device_error() == 0
    return got, want


def oracle_rows(case, rows, scale=None, max_bias=0.0, softcap=0.0):
    """Oracle on a subset of query rows (mask rows follow), full K/V."""
    scale = case.D ** -0.5 if scale is None else scale
    kt = {"f16": oracle.GGML_F16, "bf16": oracle.GGML_BF16, "q8_0": oracle.GGML_Q8_0}[case.kv]
    q = case.q_cpu.numpy()[:, :, rows]
    kc = case._np(case.k_cache_cpu)[case.s0:case.s0 + case.Bk, :, :case.n_kv]
    vc = case._np(case.v_cache_cpu)[case.s0:case.s0 + case.Bk, :, :case.n_kv]
    m = None if case.mask_cpu is None else np.ascontiguousarray(case.mask_cpu.numpy()[:, :, rows])
    s = None if case.sinks_cpu is None else case.sinks_cpu.numpy()
    return oracle.flash_attn_ext(np.ascontiguousarray(q), kc, vc, m, s, scale=scale, max_bias=max_bias,
                                 softcap=softcap, k_type=kt, v_type=kt, d=case.D, dv=case.D)


def pad256(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("S", [100, 257, 1024])
def test_lm_causal_prefill_cache_view(S):
    """qwen3-lm.h prefill: Q [128,S,16], K/V views [128,PAD(S,256),8] of a
    [128,max_seq,8] cache, causal mask [PAD(S,256), S] with -inf past each row."""
    n_kv = pad256(S)
    c = Case(42 + 1000 * 3 + S, B=1, Hq=16, Hkv=8, n_q=S, n_kv=n_kv, max_seq=4096,
             mask=lambda m: causal_mask(m, S))
    run_case(c)


def causal_mask(m, S):
    # query i (absolute position i, kv_pos = 0) sees keys 0..i
    n = m.shape[-1]
    j = torch.arange(n)
    for i in range(S):
        m[..., i, :] = torch.where(j <= i, 0.0, float("-inf"))
    return m


@pytest.mark.parametrize("S,H,Hkv", [(300, 16, 16), (600, 16, 8), (1500, 16, 16)])
def test_dit_self_attention_unmasked(S, H, Hkv):
    c = Case(42 + 1000 * 4 + S, B=2, Hq=H, Hkv=Hkv, n_q=S, n_kv=S, mask=None)
    run_case(c)


def window_mask(m, win):
    S_q, S_k = m.shape[-2], m.shape[-1]
    qi = torch.arange(S_q)[:, None]
    kj = torch.arange(S_k)[None, :]
    m[...] = torch.where((qi - kj).abs() <= win, 0.0, float("-inf"))
    return m


@pytest.mark.parametrize("S,win", [(700, 64), (1000, 128)])
def test_dit_self_attention_window(S, win):
    c = Case(42 + 1000 * 4 + 7 * S + win, B=2, Hq=16, Hkv=16, n_q=S, n_kv=S, mask=lambda m: window_mask(m, win),
             m_batch=2)
    run_case(c)


def padding_mask(valid):
    def f(m):
        for b in range(m.shape[0]):
            m[b, :, :, valid[b]:] = float("-inf")
        return m
    return f


@pytest.mark.parametrize("S,enc,valid", [(1000, 512, (461, 400)), (300, 238, (238, 200))])
def test_dit_cross_attention_padding(S, enc, valid):
    c = Case(42 + 1000 * 5 + S, B=2, Hq=16, Hkv=16, n_q=S, n_kv=enc, mask=padding_mask(valid), m_batch=2)
    run_case(c)


@pytest.mark.parametrize("n_q,n_kv", [(65, 1), (129, 130), (250, 127), (333, 1000)])
def test_ragged_shapes(n_q, n_kv):
    c = Case(42 + n_q * 7 + n_kv, B=1, Hq=4, Hkv=2, n_q=n_q, n_kv=n_kv, mask="random")
    run_case(c)


@pytest.mark.parametrize("lo,hi,scale", [(0.05, 1.0, 0.3), (1.0, 3.0, 0.5)])
def test_running_max_jumps_inside_tiles(lo, hi, scale):
    """Scores whose maximum jumps by more than 2^8 (log2 units) from the first
    64-key half of a tile to the second, in nearly every row: the first half's
    stored P, the row sum and O must all be rescaled.  Q is made exactly
    representable in f16 so that the check isolates the softmax rescaling
    from the Q -> f16 operand rounding, whose error grows with the score
    magnitude (up to ~100 log2 units here) for every F16 K/V implementation."""
    c = Case(61, B=1, Hq=8, Hkv=8, n_q=300, n_kv=700, mask=None)
    c.q_cpu = c.q_cpu.half().float()
    k = c.k_cache_cpu.float()
    j = torch.arange(k.shape[2])
    k[:, :, (j % 128) < 64] *= lo
    k[:, :, (j % 128) >= 64] *= hi
    c.k_cache_cpu = k.half()
    c.to("cuda")
    run_case(c, scale=scale)


def test_tail_units_split_over_key_ranges():
    """160 work units (16 row-tile pairs x 10 heads) on 148 SMs: the 12 of the
    last wave are each cut into two key ranges of 16 key tiles whose partial
    results a combine kernel merges, with the sink added once in the merge.
    The split units are pair 0 (rows 0-255) of every head and pair 1 of two."""
    c = Case(71, B=1, Hq=10, Hkv=10, n_q=4096, n_kv=4096, mask=None, sinks=True)
    run_case(c, rows=[0, 1, 77, 128, 255, 256, 300, 511, 2048, 4095])
    assert acefa.last_launch_count() == 2  # attention, combine


def test_sinks_softcap_alibi_dense():
    c = Case(4500, B=2, Hq=8, Hkv=4, n_q=200, n_kv=300, mask="random", sinks=True)
    run_case(c, max_bias=8.0, softcap=20.0)


def test_per_head_mask_without_classes():
    c = Case(4600, B=2, Hq=8, Hkv=2, n_q=100, n_kv=400, mask="random", m_heads=8, m_batch=1, mask_pad=9)
    run_case(c)


def test_fully_masked_rows_dense():
    def mk(m):
        m[:, :, 5, :] = float("-inf")
        m[:, :, 150:, :] = float("-inf")
        m[:, :, 10, 300:] = float("-inf")
        return m

    c = Case(4700, B=1, Hq=4, Hkv=4, n_q=200, n_kv=333, mask=mk)
    got, _ = run_case(c)
    assert np.all(got[:, 5] == 0.0) and np.all(got[:, 150:] == 0.0)


def test_mask_indexing_bit_exact_dense():
    n_kv, D = 128, 128
    c = Case(4800, B=2, Hq=4, Hkv=2, n_q=100, n_kv=n_kv, D=D, mask="random", m_heads=1, m_batch=2)
    c.q_cpu.zero_()
    c.q.zero_()
    c.v_cache_cpu[:] = torch.eye(n_kv, D).half()
    c.v_cache.copy_(c.v_cache_cpu)
    got = c.gpu()
    assert acefa.last_path() == 2
    m = c.mask_cpu.float().numpy()
    for b in range(2):
        for h in range(4):
            vis = np.isfinite(m[b, 0, :100, :n_kv])
            nz = got[b, :, h, :n_kv] != 0.0
            assert np.array_equal(vis, nz), (b, h)


@pytest.mark.parametrize("S", [6000])
def test_full_size_dit_config4_sampled_rows(S):
    """BASELINE config 4 at full size (S=6000, B=2, 16x128, window and padding
    variants): every output row is computed, a seeded sample is checked."""
    rng = np.random.default_rng(42 + 1000 * 4)
    rows = np.sort(rng.choice(S, 48, replace=False))
    rows = np.unique(np.concatenate([rows, [0, 127, 128, S - 1]]))
    c = Case(42 + 1000 * 4 + 1, B=2, Hq=16, Hkv=16, n_q=S, n_kv=S, mask=None)
    run_case(c, rows=rows)
    cw = Case(42 + 1000 * 4 + 2, B=2, Hq=16, Hkv=16, n_q=S, n_kv=S, mask=lambda m: window_mask(m, 128), m_batch=1)
    run_case(cw, rows=rows)
    cx = Case(42 + 1000 * 4 + 3, B=2, Hq=16, Hkv=16, n_q=S, n_kv=512, mask=padding_mask((461, 461)), m_batch=2)
    run_case(cx, rows=rows)


def test_full_size_prefill_config3_sampled_rows():
    """Qwen3-1.7B causal prefill, 16/8 heads, S=4096, batch 2
    (the two CFG sequences in one call), unit-RMS Q/K rows."""
    S = 4096
    rng = np.random.default_rng(42 + 1000 * 3)
    rows = np.unique(np.concatenate([np.sort(rng.choice(S, 40, replace=False)), [0, 1, 255, 256, S - 1]]))
    c = Case(42 + 1000 * 3 + 9, B=2, Hq=16, Hkv=8, n_q=S, n_kv=S, mask=lambda m: causal_mask(m, S), m_batch=1)
    # QK-norm: unit-RMS rows
    c.q_cpu = c.q_cpu / c.q_cpu.pow(2).mean(-1, keepdim=True).sqrt()
    kf = c.k_cache_cpu.float()
    c.k_cache_cpu = (kf / kf.pow(2).mean(-1, keepdim=True).sqrt()).half()
    c.to("cuda")
    run_case(c, rows=rows)


def test_binary_mask_rows_with_holes():
    """0 / -inf masks whose rows are single runs take arithmetic visibility
    (the classify pass records each row's run); rows with holes, or with a
    finite non-zero entry, keep reading the mask.  Mixed in one mask, over
    several key chunks (n_kv 2300 = 18 key tiles, chunks of 8), both kinds
    must meet the tolerance, and a row that is one run in every chunk but
    broken across chunks must not pass as a run."""
    n_q, n_kv = 256, 2300

    def mk(m):
        g = torch.Generator().manual_seed(4900)
        m[:] = float("-inf")
        for i in range(n_q):
            a = int(torch.randint(0, n_kv - 64, (1,), generator=g))
            b = int(torch.randint(a + 1, n_kv + 1, (1,), generator=g))
            m[:, :, i, a:b] = 0.0
            if i % 3 == 1 and b - a > 4:  # a hole: not a run any more
                h = int(torch.randint(a + 1, b - 1, (1,), generator=g))
                m[:, :, i, h] = float("-inf")
            if i % 7 == 2:  # one run per chunk, two runs in the row
                m[:, :, i, :] = float("-inf")
                m[:, :, i, 100:900] = 0.0
                m[:, :, i, 1500:2000] = 0.0
            if i % 11 == 5:  # a finite non-zero entry: not binary
                m[:, :, i, min(b, n_kv - 1)] = -2.5
        return m

    c = Case(4901, B=2, Hq=8, Hkv=4, n_q=n_q, n_kv=n_kv, mask=mk, m_batch=1)
    assert_close(c.gpu(), c.oracle(), what="binary mask rows with holes")


# ---------------------------------------------------------------------------
# BF16 and Q8_0 K/V on the tcgen05 path: BF16 tiles converted to F16 in
# shared memory, Q8_0 rows staged raw and dequantised (f16(d * q)) by warps
# 2-3 before the MMAs read them.

@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
@pytest.mark.parametrize("S,H,Hkv", [(300, 16, 16), (600, 16, 8)])
def test_dense_bf16_q8_unmasked(kv, S, H, Hkv):
    c = Case(42 + 1000 * 4 + S + 7, B=2, Hq=H, Hkv=Hkv, n_q=S, n_kv=S, kv=kv, mask=None)
    run_case(c)


@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
@pytest.mark.parametrize("n_q,n_kv", [(129, 130), (250, 127), (333, 1000), (512, 515)])
def test_dense_bf16_q8_ragged_masked(kv, n_q, n_kv):
    """Ragged key counts (half tiles of 64 keys partly or wholly past n_kv),
    random masks with -inf and finite entries, GQA 2."""
    c = Case(42 + n_q * 11 + n_kv, B=1, Hq=4, Hkv=2, n_q=n_q, n_kv=n_kv, kv=kv, mask="random")
    run_case(c)


@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
def test_dense_bf16_q8_causal_prefill_cache_view(kv):
    """The reference's prefill over its KV cache: views [128, PAD(S,256), 8] of a
    cache of max_seq rows at set 2, causal mask."""
    S = 300
    c = Case(42 + 3000 + S, B=1, Hq=16, Hkv=8, n_q=S, n_kv=512, kv=kv, max_seq=2560, s0=2,
             mask=lambda m: causal_mask(m, S))
    run_case(c)


@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
def test_dense_bf16_q8_split_tail_units(kv):
    """Unmasked node whose last-wave units are split over key ranges (the
    combine kernel merges them)."""
    c = Case(72, B=1, Hq=10, Hkv=10, n_q=4096, n_kv=4096, kv=kv, mask=None, sinks=True)
    run_case(c, rows=[0, 1, 255, 256, 2048, 4095])


def test_full_size_dit_bf16_sampled_rows():
    """BASELINE config 4 with BF16 inputs: DiT self-attention S = 6000, B = 2,
    16 x 128, and the cross-attention padding case."""
    S = 6000
    rng = np.random.default_rng(42 + 1000 * 4 + 5)
    rows = np.unique(np.concatenate([np.sort(rng.choice(S, 40, replace=False)), [0, 127, 128, S - 1]]))
    c = Case(42 + 1000 * 4 + 11, B=2, Hq=16, Hkv=16, n_q=S, n_kv=S, kv="bf16", mask=None)
    run_case(c, rows=rows)
    cx = Case(42 + 1000 * 4 + 13, B=2, Hq=16, Hkv=16, n_q=S, n_kv=512, kv="bf16", mask=padding_mask((461, 461)),
              m_batch=2)
    run_case(cx, rows=rows)


# ---- D = 64 on the tcgen05 path: one 64-dim box per K/V tile, four S k-steps,
# an N = 64 PV MMA.

@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
@pytest.mark.parametrize("S,H,Hkv", [(300, 16, 16), (600, 16, 8)])
def test_dense_d64_unmasked(kv, S, H, Hkv):
    c = Case(42 + 6400 + S + H + Hkv, B=2, Hq=H, Hkv=Hkv, n_q=S, n_kv=S, D=64, kv=kv, mask=None)
    run_case(c)


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
@pytest.mark.parametrize("n_q,n_kv", [(129, 130), (333, 1000)])
def test_dense_d64_ragged_masked(kv, n_q, n_kv):
    c = Case(42 + 6401 + n_q + n_kv, B=1, Hq=4, Hkv=2, n_q=n_q, n_kv=n_kv, D=64, kv=kv, mask="random")
    run_case(c)


def test_dense_d64_causal_cache_view_and_split_tail():
    S = 300
    c = Case(42 + 6402, B=1, Hq=16, Hkv=8, n_q=S, n_kv=512, D=64, max_seq=2560, s0=1,
             mask=lambda m: causal_mask(m, S))
    run_case(c)
    c2 = Case(42 + 6403, B=1, Hq=10, Hkv=10, n_q=4096, n_kv=4096, D=64, mask=None, sinks=True)
    run_case(c2, rows=[0, 1, 255, 256, 2048, 4095])
    assert acefa.last_launch_count() == 2  # attention, combine


def test_dense_d64_sinks_softcap_alibi():
    c = Case(42 + 6404, B=2, Hq=8, Hkv=4, n_q=200, n_kv=300, D=64, mask="random", sinks=True)
    run_case(c, max_bias=8.0, softcap=20.0)


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (16, 16)])
def test_q_staging_tma_and_thread_loads_agree(Hq, Hkv):
    """The dense kernel stages a unit's f32 Q rows by TMA when a tensor map can
    describe them (16-B aligned base and strides, 128 % G == 0) and by
    per-thread loads otherwise.  Both convert the same values, so a Q copied to
    a 4-byte offset (thread loads) and a head-interleaved Q (the layout of a
    ggml_permute of the projection: head stride below query stride, TMA) give
    outputs bit-identical to the contiguous Q."""
    c = Case(4242 + Hq + Hkv, B=2, Hq=Hq, Hkv=Hkv, n_q=700, n_kv=900, mask="random")
    got, _ = run_case(c)
    buf = torch.empty(c.q.numel() + 1, device="cuda")
    q_off = buf[1:].view(c.q.shape)
    q_off.copy_(c.q)
    q_perm = c.q.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)  # (B, Hq, n_q, D), heads innermost
    assert q_perm.stride(1) < q_perm.stride(2)
    for q in (q_off, q_perm):
        out = acefa.Op(q, c.k, c.v, mask=c.mask, kv_type=c.kv_type)()
        torch.cuda.synchronize()
        assert acefa.last_path() == 2
        assert np.array_equal(out.cpu().numpy().view(np.uint32), got.view(np.uint32))
    assert acefa.device_error() == 0


def test_q_staging_group_not_dividing_the_row_tile():
    """G = 3 (24 query heads over 8 KV heads): 128 % G != 0, so Q goes through
    the per-thread loads; parity with the oracle."""
    c = Case(4343, B=1, Hq=24, Hkv=8, n_q=300, n_kv=500, mask="random")
    run_case(c)


@pytest.mark.parametrize("mask", ["random", None])
def test_bf16_conversion_pass_and_converter_warps_agree(mask):
    """BF16 K/V: with room in the workspace one pass converts them to F16 copies
    that the F16 kernel reads; without it the kernel's converter warps convert
    each staged tile.  Both round bf16 -> f32 -> f16 to nearest even, so the
    outputs are bit-identical (and the pass is one extra launch)."""
    c = Case(5151, B=2, Hq=16, Hkv=8, n_q=600, n_kv=700, kv="bf16", mask=mask)
    op = c.op()
    conv = (2 * c.Bk * c.Hkv * c.n_kv * c.D * 2 + 255) // 256 * 256
    assert op.ws_bytes >= conv
    full = op().clone()
    torch.cuda.synchronize()
    assert acefa.last_path() == 2
    n_full = acefa.last_launch_count()
    op.workspace = op.workspace[: max(op.ws_bytes - conv, 256)]
    part = op().clone()
    torch.cuda.synchronize()
    assert acefa.last_launch_count() == n_full - 1
    assert torch.equal(full.view(torch.int32), part.view(torch.int32))
    assert_close(part.cpu().numpy(), c.oracle(), what="bf16 converter warps")
    assert acefa.device_error() == 0


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (16, 16)])
def test_output_tma_stores_and_lane_stores_agree(Hq, Hkv):
    """Output rows leave the dense kernel by TMA stores when a tensor map can
    describe the destination (16-B aligned base and strides, 32 % G == 0, no
    mirrors) and by per-lane stores otherwise: an output at a 4-byte offset
    takes the second route and must hold the same bits.  Ragged row count."""
    c = Case(4545 + Hq + Hkv, B=2, Hq=Hq, Hkv=Hkv, n_q=333, n_kv=500, mask="random")
    got, _ = run_case(c)
    buf = torch.empty(got.size + 1, device="cuda")
    out_off = buf[1:].view(got.shape)
    acefa.Op(c.q, c.k, c.v, mask=c.mask, kv_type=c.kv_type, out=out_off)()
    torch.cuda.synchronize()
    assert acefa.last_path() == 2
    assert np.array_equal(out_off.cpu().numpy().view(np.uint32), got.view(np.uint32))
    assert acefa.device_error() == 0


def test_tma_q_and_output_with_padded_strides():
    """Q and the output as views of padded buffers (every stride a multiple
    of 16 B, none tight): the Q copy and the output stores still go by TMA,
    and the results are bit-identical to the tight layouts."""
    c = Case(4646, B=2, Hq=16, Hkv=8, n_q=300, n_kv=400, mask="random")
    got, _ = run_case(c)
    D = c.D
    qbuf = torch.zeros(c.B, c.Hq + 1, c.n_q + 3, D + 4, device="cuda")
    q_pad = qbuf[:, :c.Hq, :c.n_q, :D]
    q_pad.copy_(c.q)
    obuf = torch.zeros(c.B, c.n_q + 1, c.Hq + 2, D + 8, device="cuda")
    o_pad = obuf[:, :c.n_q, :c.Hq, :D]
    acefa.Op(q_pad, c.k, c.v, mask=c.mask, kv_type=c.kv_type, out=o_pad)()
    torch.cuda.synchronize()
    assert acefa.last_path() == 2
    assert np.array_equal(o_pad.cpu().numpy().view(np.uint32), got.view(np.uint32))
    # the padding around the output is untouched
    rest = obuf.clone()
    rest[:, :c.n_q, :c.Hq, :D] = 0
    assert torch.count_nonzero(rest) == 0
    assert acefa.device_error() == 0


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
def test_dense_kv_shared_by_batches(kv):
    """K/V with one batch shared by two query batches (ggml: K ne3 = 1, Q ne3 =
    2; query batch b reads K/V batch b / 2): the TMA Q / output maps, the BF16
    copies and the Q8_0 staging all index the K/V batch by bk = b / rk3."""
    c = Case(4747 + len(kv), B=2, Bk=1, Hq=16, Hkv=8, n_q=260, n_kv=390, kv=kv, mask="random", m_batch=2)
    run_case(c)
