"""GPU parity of the split-KV decode path against the CPU oracle, through the
C ABI.  Tolerance (north star): FP32 output within max-abs 2e-3 and cosine
>= 0.99995 of the FP32 oracle; mask indexing bit-exact."""
import numpy as np
import pytest
import torch

import acefa
import oracle
from fa_cases import Case, assert_close, cosine

pytestmark = pytest.mark.gpu


def run_case(case, **kw):
    got = case.gpu(**kw)
    want = case.oracle(**kw)
    err = assert_close(got, want, what=str(kw))
    assert acefa.device_error() == 0
    return got, want, err


def test_config1_qwen3_0p6b_decode():
    """B=1, 1 query, Hq=16/Hkv=8, D=128, n_kv=2048, Q f32, K/V f16."""
    c = Case(42 + 1000 * 1, B=1, Hq=16, Hkv=8, n_q=1, n_kv=2048, mask="zeros")
    run_case(c)
    assert acefa.last_path() == 1


@pytest.mark.parametrize("kv", ["f16", "q8_0", "bf16"])
def test_batched_cfg_decode_views(kv):
    """qwen3-lm.h batched decode: views of consecutive sets s0.. of a
    [D, max_seq, Hkv, sets] cache, per-set valid lengths in the mask."""
    valid = [300, 301, 257, 512]
    c = Case(42 + 1000 * 2, B=4, Hq=32, Hkv=8, n_q=1, n_kv=512, kv=kv, max_seq=1024, s0=1,
             mask="valid", valid=valid)
    run_case(c)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
def test_gqa_ratios(G):
    Hkv = 2 if G <= 8 else 1
    c = Case(100 + G, B=2, Hq=Hkv * G, Hkv=Hkv, n_q=1, n_kv=700, mask="random")
    run_case(c)


@pytest.mark.parametrize("n_kv", [1, 2, 33, 63, 64, 65, 1000])
@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_ragged_kv_lengths(n_kv, kv):
    c = Case(200 + n_kv, B=1, Hq=8, Hkv=4, n_q=1, n_kv=n_kv, kv=kv, mask="zeros")
    run_case(c)


@pytest.mark.parametrize("kv", ["f16", "q8_0", "bf16"])
def test_head_dim_64(kv):
    c = Case(300, B=2, Hq=8, Hkv=2, n_q=3, n_kv=333, D=64, kv=kv, mask="random")
    run_case(c)


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_head_dim_256(kv):
    """D = 256 (F16 and BF16 K/V, on this kernel at one CTA per SM): batched
    decode over cache views with per-set lengths, GQA 2, a prefill-sized node
    with a causal mask, and sinks / softcap / ALiBi."""
    c = Case(310, B=4, Hq=8, Hkv=4, n_q=1, n_kv=700, D=256, kv=kv, max_seq=1024, s0=1, mask="valid",
             valid=[700, 333, 64, 65])
    run_case(c)
    assert acefa.last_path() == 1
    c2 = Case(311, B=1, Hq=8, Hkv=4, n_q=200, n_kv=256, D=256, kv=kv, mask="causal")
    run_case(c2)
    c3 = Case(312, B=2, Hq=8, Hkv=4, n_q=2, n_kv=300, D=256, kv=kv, mask="random", sinks=True)
    run_case(c3, max_bias=8.0, softcap=20.0)


def test_head_dim_256_refusals():
    """Q8_0 K/V and the Q prologue are refused at D = 256 (before any launch)."""
    c = Case(313, B=1, Hq=8, Hkv=4, n_q=1, n_kv=128, D=256, mask="zeros")
    q8 = acefa.quantize_q8_0(c.k.float())
    with pytest.raises(acefa.AcefaError) as e:
        acefa.Op(c.q, q8, q8, mask=c.mask, kv_type=acefa.GGML_Q8_0)()
    assert e.value.status == -2
    pro = acefa.RopeNorm(torch.ones(256, device="cuda"), 1e-6, 1.0e6, torch.zeros(1, dtype=torch.int32, device="cuda"))
    with pytest.raises(acefa.AcefaError) as e:
        acefa.Op(c.q, c.k, c.v, mask=c.mask, q_prologue=pro)()
    assert e.value.status == -3


@pytest.mark.parametrize("n_q", [2, 5, 6, 20])
def test_short_query_blocks(n_q):
    """FSQ tokenizer/detokenizer (S=5/6, no mask) and multi row-block units."""
    c = Case(400 + n_q, B=1, Hq=16, Hkv=8, n_q=n_q, n_kv=n_q + 40, mask="causal")
    run_case(c)
    c2 = Case(410 + n_q, B=1, Hq=16, Hkv=16, n_q=n_q, n_kv=n_q, mask=None)
    run_case(c2)


def test_sinks_softcap_alibi():
    c = Case(500, B=2, Hq=8, Hkv=4, n_q=2, n_kv=300, mask="random", sinks=True)
    run_case(c, max_bias=8.0, softcap=20.0)
    run_case(c, scale=0.05)


def test_mask_broadcast_and_kv_broadcast():
    # mask shared over batch (Bm = 1) and per-head (Hm = Hq); K/V shared by batch (Bk = 1)
    c = Case(600, B=3, Hq=8, Hkv=2, n_q=2, n_kv=257, Bk=1, mask="random", m_heads=8, m_batch=1, mask_pad=7)
    run_case(c)


def test_fully_masked_rows_are_zero():
    def mk(m):
        m[:, :, 1, :] = float("-inf")  # query 1 sees nothing
        m[:, :, 0, 100:] = float("-inf")
        return m

    c = Case(700, B=2, Hq=4, Hkv=2, n_q=3, n_kv=400, mask=mk)
    got, want, _ = run_case(c)
    assert np.all(got[:, 1] == 0.0)


def test_padded_window_tail_is_skipped_exactly():
    """The decode window is PAD(kv_len, 256); keys past kv_len carry -inf and
    must contribute nothing even when the cache holds huge stale values there
    (a key that leaked through would dominate the softmax)."""
    c = Case(800, B=2, Hq=16, Hkv=8, n_q=1, n_kv=768, mask="valid", valid=[513, 700])
    c.k_cache_cpu[0, :, 513:] = 60000.0
    c.v_cache_cpu[0, :, 513:] = -60000.0
    c.to("cuda")
    run_case(c)


def test_mask_indexing_bit_exact():
    """With Q = 0 every visible key gets the same weight; V = one-hot rows make
    each output lane an exact indicator of one key's visibility."""
    n_kv, D = 128, 128
    c = Case(900, B=2, Hq=4, Hkv=2, n_q=3, n_kv=n_kv, D=D, mask="random", m_heads=4, m_batch=2)
    c.q.zero_()
    c.q_cpu.zero_()
    eye = torch.eye(n_kv, D).half()
    c.v_cache_cpu[:] = eye
    c.v_cache.copy_(c.v_cache_cpu)
    got = c.gpu()
    m = c.mask_cpu.float().numpy()  # (Bm, Hm, n_q, n_kv)
    for b in range(2):
        for h in range(4):
            for i in range(3):
                vis = np.isfinite(m[b, h, i, :n_kv])
                nz = got[b, i, h, :n_kv] != 0.0
                assert np.array_equal(vis, nz), (b, h, i)


@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_full_size_layer_config2(kv):
    """One layer of BASELINE config 2 at full size: Qwen3-4B, 8 requests x CFG =
    16 sets, Hq=32/Hkv=8, KV length 8192 (max_seq 8192)."""
    c = Case(42 + 1000 * 2 + 7, B=16, Hq=32, Hkv=8, n_q=1, n_kv=8192, kv=kv, mask="zeros")
    run_case(c)


def test_cuda_graph_replay_with_new_mask():
    """Grid and workspace depend on shapes only: a captured graph replays
    correctly after the mask (valid lengths) changes in place."""
    c = Case(1000, B=4, Hq=32, Hkv=8, n_q=1, n_kv=512, mask="valid", valid=[100, 200, 300, 400])
    op = c.op()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        op(stream=s)  # warm-up outside capture
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=s):
            op(stream=s)
    for valid in ([100, 200, 300, 400], [512, 1, 256, 257]):
        m = torch.zeros(4, 1, 1, 512)
        for b in range(4):
            m[b, :, :, valid[b]:] = float("-inf")
        c.mask_cpu = m.half()
        c.mask.copy_(c.mask_cpu)
        op.out.fill_(float("nan"))
        gph.replay()
        torch.cuda.synchronize()
        assert_close(op.out.cpu().numpy(), c.oracle())
    del gph


def test_distance_to_ggml_cpu_arithmetic():
    """Report-only bound: the F32-accumulating kernel sits closer to the exact
    result than ggml-cpu's F16 accumulation, and within 2e-2 of it."""
    c = Case(1100, B=1, Hq=16, Hkv=8, n_q=1, n_kv=2048, mask="zeros")
    got = c.gpu()
    f32 = c.oracle()
    g16 = c.oracle(mode=oracle.MODE_GGML_CPU)
    assert np.abs(got - g16).max() < 2e-2
    assert np.abs(got - f32).max() <= np.abs(g16 - f32).max() + 1e-4
    assert cosine(got, g16) > 0.999


def test_decode_needs_no_workspace():
    """Split keys merge inside the thread-block cluster: the decode path runs
    with no workspace at all (NULL, 0 bytes) and gives the same result."""
    c = Case(1200, B=16, Hq=32, Hkv=8, n_q=1, n_kv=2048, mask="valid", valid=[2048 - 61 * i for i in range(16)])
    op = c.op()
    want = op().clone()
    assert acefa.last_launch_count() == 1 and acefa.last_path() == 1
    op.out.fill_(float("nan"))
    st = op.lib.acefa_flash_attn_ext(
        acefa._ref(op.tq), acefa._ref(op.tk), acefa._ref(op.tv), acefa._ref(op.tm), None, acefa._ref(op.td),
        op.scale, 0.0, 0.0, op.prec, None, None, 0)
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(op.out, want)
    assert_close(want.cpu().numpy(), c.oracle())


def test_workspace_too_small_is_rejected():
    """The dense path's mask class table lives in the workspace."""
    c = Case(1201, B=1, Hq=16, Hkv=8, n_q=600, n_kv=700, mask="random")
    op = c.op()
    assert op.ws_bytes >= 256
    op.workspace = op.workspace[: max(op.ws_bytes // 2, 1)]
    with pytest.raises(acefa.AcefaError) as e:
        op()
    assert e.value.status == -5


@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_very_long_kv_single_set(kv):
    """Long contexts on the split-KV kernel: 2 sets x 160,000 keys (2,500
    tiles per unit over clusters of 8), a validity mask cutting each set at a
    different length."""
    n = 160_000
    c = Case(1700, B=2, Hq=16, Hkv=8, n_q=1, n_kv=n, kv=kv, mask="valid", valid=[n, 99_991])
    run_case(c)
    assert acefa.last_path() == 1


def test_query_heavy_node_past_dense_key_limit():
    """A prefill-shaped node (256 query rows per K/V head) with more keys than
    the dense kernel's class table holds (70,000 > 65,536) runs on the split-KV
    kernel; sampled rows against the oracle."""
    c = Case(1701, B=1, Hq=2, Hkv=1, n_q=128, n_kv=70_000, mask="random")
    got = c.gpu()
    assert acefa.last_path() == 1
    rows = [0, 1, 63, 64, 127]
    from test_dense_gpu import oracle_rows
    want = oracle_rows(c, rows)
    assert_close(got[:, rows], want, what="70k keys, sampled rows")
    assert acefa.device_error() == 0
