"""The attention prologue on the GPU: QK-norm (RMSNorm times a weight) and
RoPE NEOX (src/qwen3-lm.h:423-431, src/dit-graph.h:181-197) fused into

  * the attention kernels' Q load (acefa_op_ext::q_prologue, decode and dense),
  * the fused KV-cache append of a decode step (acefa_op_ext::k_prologue),
  * acefa_kv_prologue, one pass that prepares K and V for the dense path.

The checker is the oracle: ora_rope_norm (pinned against the Qwen3 model
definition, tests/test_oracle.py) applied to the raw rows, then the attention
oracle on the results.  Outputs meet the north-star tolerance; prepared K/V
rows agree with the oracle's rows after the same F16/BF16 rounding to within
one unit in the last place (the f32 prologue differs from the oracle's by
summation order and the libm sin/cos, so a value next to a rounding boundary
may round the other way)."""
import numpy as np
import pytest
import torch

import acefa
import oracle
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu

THETA, EPS = 1.0e6, 1e-6


def _weights(D, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.25 * torch.randn(D, generator=g)).float()


def _ora_rows(x, w, positions_of_row):
    """oracle.rope_norm over x (..., D) with one position per row."""
    D = x.shape[-1]
    pos = np.asarray(positions_of_row, dtype=np.int32).reshape(-1)
    return oracle.rope_norm(x.reshape(-1, D), w, EPS, THETA, pos).reshape(x.shape)


def _q_positions(B, Hq, n_q, pos):
    """Position of each row of Q (B, Hq, n_q, D): pos[iq + b * n_q]."""
    idx = (np.arange(B)[:, None, None] * n_q + np.arange(n_q)[None, None, :]).repeat(Hq, axis=1)
    return pos[idx]


def _ulp_close(got, want, dtype):
    """Rows rounded to f16 / bf16: equal to within one unit in the last place,
    or, for values that came out of a cancellation in the rotation (a small
    difference of two products), within the f32 error of those products: a few
    f32 ulps of the row's largest value."""
    g = got.float().cpu().numpy()
    w = torch.from_numpy(want).to(dtype).float().numpy()
    rel = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    # one step of the coarser of the two values' binades (a pair straddling a
    # power of two is one step apart in the upper binade)
    tol = np.maximum(np.maximum(np.abs(w), np.abs(g)), 2.0 ** -14) * rel * 1.01
    row_max = np.abs(want).max(axis=-1, keepdims=True)
    tol = np.maximum(tol, 8 * 2.0 ** -23 * row_max)
    bad = np.abs(g - w) > tol
    assert not bad.any(), f"{bad.sum()} values differ by more than one ulp (max {np.abs(g - w).max()})"


def _q_case(c, pos_np, w):
    """The oracle's view of the case: Q after the prologue."""
    qn = _ora_rows(c.q_cpu.numpy(), w.numpy(), _q_positions(c.B, c.Hq, c.n_q, pos_np))
    c.q_cpu = torch.from_numpy(qn)
    return c


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("mask", [None, "causal"])
def test_dense_q_prologue(mask, D):
    # DiT-like (unmasked) and prefill-like (causal, GQA 2) nodes on the dense path
    Hq, Hkv = (16, 16) if mask is None else (16, 8)
    c = Case(101 + D, B=2, Hq=Hq, Hkv=Hkv, n_q=300, n_kv=300, D=D, mask=mask)
    w = _weights(D, 1)
    pos = np.tile(np.arange(300, dtype=np.int32) + 1000, 2)  # positions[iq + b * n_q]
    pro = acefa.RopeNorm(w.cuda(), EPS, THETA, torch.from_numpy(pos).cuda())
    got = acefa.Op(c.q, c.k, c.v, mask=c.mask, q_prologue=pro)()
    torch.cuda.synchronize()
    assert acefa.last_path() == 2
    assert_close(got.cpu().numpy(), _q_case(c, pos, w).oracle(), what="dense q prologue")


@pytest.mark.parametrize("kv,D", [("bf16", 128), ("q8_0", 128), ("bf16", 64), ("q8_0", 64)])
def test_dense_q_prologue_bf16_q8_0(kv, D):
    # the prologue instances of the dense kernel with converted K/V (causal, GQA 2)
    c = Case(131 + D, B=2, Hq=16, Hkv=8, n_q=300, n_kv=300, D=D, kv=kv, mask="causal")
    w = _weights(D, 3)
    pos = np.tile(np.arange(300, dtype=np.int32) + 50, 2)
    pro = acefa.RopeNorm(w.cuda(), EPS, THETA, torch.from_numpy(pos).cuda())
    got = acefa.Op(c.q, c.k, c.v, mask=c.mask, kv_type=c.kv_type, q_prologue=pro)()
    torch.cuda.synchronize()
    assert acefa.last_path() == 2
    assert_close(got.cpu().numpy(), _q_case(c, pos, w).oracle(), what=f"dense q prologue {kv} D{D}")


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
def test_decode_q_prologue(kv):
    # batched decode: one query per set, position kv_pos of its set
    kv_pos = np.array([0, 350, 699, 511], dtype=np.int32)
    c = Case(102, B=4, Hq=32, Hkv=8, n_q=1, n_kv=704, kv=kv, mask="valid", valid=list(kv_pos + 1))
    w = _weights(128, 2)
    pro = acefa.RopeNorm(w.cuda(), EPS, THETA, torch.from_numpy(kv_pos).cuda())
    got = acefa.Op(c.q, c.k, c.v, mask=c.mask, kv_type=c.kv_type, q_prologue=pro)()
    torch.cuda.synchronize()
    assert acefa.last_path() == 1
    assert_close(got.cpu().numpy(), _q_case(c, kv_pos, w).oracle(), what=f"decode q prologue {kv}")


def test_decode_short_queries_prologue_norm_only():
    # several queries per row block (FSQ-encoder-like), RMSNorm without RoPE
    c = Case(103, B=2, Hq=16, Hkv=16, n_q=6, n_kv=6, mask=None)
    w = _weights(128, 3)
    got = acefa.Op(c.q, c.k, c.v, q_prologue=acefa.RopeNorm(w.cuda(), EPS, 0.0, None))()
    torch.cuda.synchronize()
    qn = oracle.rope_norm(c.q_cpu.numpy().reshape(-1, 128), w.numpy(), EPS, 0.0, None).reshape(c.q_cpu.shape)
    c.q_cpu = torch.from_numpy(qn)
    assert_close(got.cpu().numpy(), c.oracle(), what="norm-only prologue")


@pytest.mark.parametrize("kv", ["f16", "bf16", "q8_0"])
def test_decode_step_fully_fused(kv):
    """One LM decode step: raw Q and raw new K row in, the cache row written
    as RoPE(RMSNorm(k_new)), attention over the updated cache out."""
    B, Hq, Hkv, n_kv = 4, 32, 8, 704
    kv_pos = np.array([0, 350, 699, 511], dtype=np.int32)
    c = Case(104, B=B, Hq=Hq, Hkv=Hkv, n_q=1, n_kv=n_kv, kv=kv, mask="valid", valid=list(kv_pos + 1))
    g = torch.Generator().manual_seed(105)
    k_new = torch.randn(B, Hkv, 1, 128, generator=g) * 2.0
    v_new = torch.randn(B, Hkv, 1, 128, generator=g)
    wq, wk = _weights(128, 4), _weights(128, 5)
    pos_t = torch.from_numpy(kv_pos).cuda()
    op = acefa.Op(c.q, c.k, c.v, mask=c.mask, kv_type=c.kv_type, k_new=k_new.cuda(), v_new=v_new.cuda(),
                  pos=torch.from_numpy(kv_pos.astype(np.int64)).cuda(),
                  q_prologue=acefa.RopeNorm(wq.cuda(), EPS, THETA, pos_t),
                  k_prologue=acefa.RopeNorm(wk.cuda(), EPS, THETA, pos_t))
    got = op()
    torch.cuda.synchronize()
    assert acefa.device_error() == 0
    # the written rows: the oracle's prologue of k_new, same conversion
    kn = _ora_rows(k_new.numpy(), wk.numpy(), np.repeat(kv_pos, Hkv))
    for b, p in enumerate(kv_pos):
        row = c.k_cache[b, :, p].cpu()
        if kv == "q8_0":
            deq = acefa.dequantize_q8_0(row).numpy()
            step = np.abs(kn[b, :, 0]).reshape(Hkv, -1, 32).max(axis=2, keepdims=True) / 127.0
            # within one quantisation step of the oracle's row (its own rounding
            # is half a step; the f32 prologues may straddle a boundary)
            assert (np.abs(deq.reshape(Hkv, -1, 32) - kn[b, :, 0].reshape(Hkv, -1, 32)) <= step * 1.01 + 1e-6).all()
            # V rows: exactly the plain quantiser's bytes
            assert torch.equal(c.v_cache[b, :, p].cpu(), acefa.quantize_q8_0(v_new[b, :, 0]))
        else:
            dt = torch.float16 if kv == "f16" else torch.bfloat16
            _ulp_close(row, kn[b, :, 0], dt)
            assert torch.equal(c.v_cache[b, :, p].cpu(), v_new[b, :, 0].to(dt))
    # the output: attention over the cache as written, Q through the oracle's prologue
    c.k_cache_cpu, c.v_cache_cpu = c.k_cache.cpu(), c.v_cache.cpu()
    assert_close(got.cpu().numpy(), _q_case(c, kv_pos, wq).oracle(), what=f"fused decode step {kv}")


@pytest.mark.parametrize("dst", ["f16", "bf16"])
def test_kv_prologue_matches_oracle(dst):
    # K/V as the DiT's projections leave them: [D, H, S, N] f32, read through the
    # permuted view [D, S, H, N] (torch (N, H, S, D) with strides of (N, S, H, D))
    N, H, S, D = 2, 8, 333, 128
    g = torch.Generator().manual_seed(106)
    k_raw = (torch.randn(N, S, H, D, generator=g) * 2.0).cuda()
    v_raw = torch.randn(N, S, H, D, generator=g).cuda()
    k_src, v_src = k_raw.permute(0, 2, 1, 3), v_raw.permute(0, 2, 1, 3)
    dt = torch.float16 if dst == "f16" else torch.bfloat16
    k_dst = torch.empty(N, H, S, D, dtype=dt, device="cuda")
    v_dst = torch.empty(N, H, S, D, dtype=dt, device="cuda")
    w = _weights(D, 7)
    pos = np.tile(np.arange(S, dtype=np.int32), N)
    acefa.kv_prologue(k_src, k_dst, v_src, v_dst, acefa.RopeNorm(w.cuda(), EPS, THETA, torch.from_numpy(pos).cuda()))
    torch.cuda.synchronize()
    kp = np.arange(S)[None, None, :].repeat(H, axis=1).repeat(N, axis=0)
    want = _ora_rows(k_src.cpu().contiguous().numpy(), w.numpy(), kp)
    _ulp_close(k_dst, want, dt)
    assert torch.equal(v_dst.cpu(), v_src.cpu().to(dt))


def test_dit_layer_prologue_then_attention():
    """DiT self-attention with every prologue fused: acefa_kv_prologue for K/V,
    the Q prologue inside the dense kernel."""
    N, H, S, D = 2, 16, 600, 128
    g = torch.Generator().manual_seed(107)
    q_raw = torch.randn(N, H, S, D, generator=g) * 2.0
    k_raw = torch.randn(N, H, S, D, generator=g) * 2.0
    v_raw = torch.randn(N, H, S, D, generator=g)
    wq, wk = _weights(D, 8), _weights(D, 9)
    pos = np.tile(np.arange(S, dtype=np.int32), N)
    pos_t = torch.from_numpy(pos).cuda()
    k16 = torch.empty(N, H, S, D, dtype=torch.float16, device="cuda")
    v16 = torch.empty_like(k16)
    acefa.kv_prologue(k_raw.cuda(), k16, v_raw.cuda(), v16, acefa.RopeNorm(wk.cuda(), EPS, THETA, pos_t))
    got = acefa.Op(q_raw.cuda(), k16, v16, q_prologue=acefa.RopeNorm(wq.cuda(), EPS, THETA, pos_t))()
    torch.cuda.synchronize()
    rows = np.arange(S)[None, None, :].repeat(H, axis=1).repeat(N, axis=0)
    qn = _ora_rows(q_raw.numpy(), wq.numpy(), rows)
    want = oracle.flash_attn_ext(qn, k16.cpu().numpy(), v16.cpu().numpy(), None, None, scale=D ** -0.5)
    assert_close(got.cpu().numpy(), want, what="DiT layer with fused prologues")


def test_prologue_refusals():
    c = Case(108, B=1, Hq=8, Hkv=8, n_q=1, n_kv=64, mask=None)
    w = _weights(128, 10).cuda()
    with pytest.raises(acefa.AcefaError) as e:  # RoPE without positions
        acefa.Op(c.q, c.k, c.v, q_prologue=acefa.RopeNorm(w, EPS, THETA, None))()
    assert e.value.status == -1
    with pytest.raises(acefa.AcefaError) as e:  # a K prologue needs the appended row
        acefa.Op(c.q, c.k, c.v, k_prologue=acefa.RopeNorm(w, EPS, 0.0, None))()
    assert e.value.status == -3
