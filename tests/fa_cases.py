"""Shared helpers for the GPU parity tests: seeded ggml-layout operands, the
oracle call on the same bytes, and the north-star tolerance check."""
from __future__ import annotations

import numpy as np
import torch

import acefa
import oracle

# North-star tolerance (FP32 output vs the FP32 CPU oracle).
MAX_ABS = 2e-3
MIN_COS = 0.99995


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(got: np.ndarray, want: np.ndarray, max_abs=MAX_ABS, min_cos=MIN_COS, what=""):
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = float(np.abs(got - want).max())
    cos = cosine(got, want)
    assert err <= max_abs and cos >= min_cos, f"{what}: max_abs={err:.3e} cos={cos:.7f}"
    return err, cos


class Case:
    """ggml_flash_attn_ext operands in torch order, built on `device`.

    K/V live in a cache [D, max_seq, Hkv, sets] (torch (sets, Hkv, max_seq, D))
    and the op reads the view of n_kv rows starting at set s0, exactly like
    qwen3-lm.h's batched decode views."""

    def __init__(self, seed, B, Hq, Hkv, n_q, n_kv, D=128, kv="f16", Bk=None, max_seq=None, s0=0,
                 mask="zeros", mask_pad=0, m_heads=1, m_batch=None, valid=None, device="cuda",
                 sinks=False, q_scale=1.0):
        g = torch.Generator().manual_seed(seed)
        Bk = B if Bk is None else Bk
        max_seq = n_kv if max_seq is None else max_seq
        self.B, self.Hq, self.Hkv, self.n_q, self.n_kv, self.D, self.Bk = B, Hq, Hkv, n_q, n_kv, D, Bk
        self.kv = kv
        q = torch.randn(B, Hq, n_q, D, generator=g) * q_scale
        kf = torch.randn(s0 + Bk, Hkv, max_seq, D, generator=g)
        vf = torch.randn(s0 + Bk, Hkv, max_seq, D, generator=g)
        if kv == "f16":
            kc, vc = kf.half(), vf.half()
            self.kv_type = None
        elif kv == "bf16":
            kc, vc = kf.bfloat16(), vf.bfloat16()
            self.kv_type = None
        elif kv == "q8_0":
            kc, vc = acefa.quantize_q8_0(kf), acefa.quantize_q8_0(vf)
            self.kv_type = acefa.GGML_Q8_0
        else:
            raise ValueError(kv)
        self.q_cpu = q.contiguous()
        self.k_cache_cpu, self.v_cache_cpu = kc.contiguous(), vc.contiguous()
        # mask [n_kv + mask_pad, n_q, m_heads, m_batch]
        mb = B if m_batch is None else m_batch
        self.mask_cpu = None
        if mask is not None:
            m = torch.zeros(mb, m_heads, n_q, n_kv + mask_pad)
            if mask == "zeros":
                pass
            elif mask == "valid":
                for b in range(mb):
                    m[b, :, :, valid[b]:] = float("-inf")
            elif mask == "causal":
                # query i sits at absolute position n_kv - n_q + i
                for i in range(n_q):
                    m[:, :, i, n_kv - n_q + i + 1:] = float("-inf")
            elif mask == "random":
                r = torch.rand(mb, m_heads, n_q, n_kv + mask_pad, generator=g)
                m = torch.where(r < 0.3, torch.full_like(m, float("-inf")),
                                torch.randn(m.shape, generator=g) * 0.5)
            elif callable(mask):
                m = mask(m)
            else:
                raise ValueError(mask)
            self.mask_cpu = m.half().contiguous()
        self.sinks_cpu = torch.randn(Hq, generator=g) if sinks else None
        self.s0 = s0
        self.to(device)

    def to(self, device):
        self.device = device
        self.q = self.q_cpu.to(device)
        self.k_cache = self.k_cache_cpu.to(device)
        self.v_cache = self.v_cache_cpu.to(device)
        self.k = self.k_cache[self.s0:self.s0 + self.Bk, :, :self.n_kv]
        self.v = self.v_cache[self.s0:self.s0 + self.Bk, :, :self.n_kv]
        self.mask = self.mask_cpu.to(device) if self.mask_cpu is not None else None
        self.sinks = self.sinks_cpu.to(device) if self.sinks_cpu is not None else None
        return self

    def _np(self, t):
        if t is None:
            return None
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16)
        return t.numpy()

    def oracle(self, scale=None, max_bias=0.0, softcap=0.0, mode=oracle.MODE_F32):
        scale = self.D ** -0.5 if scale is None else scale
        kt = {"f16": oracle.GGML_F16, "bf16": oracle.GGML_BF16, "q8_0": oracle.GGML_Q8_0}[self.kv]
        kc = self._np(self.k_cache_cpu)[self.s0:self.s0 + self.Bk, :, :self.n_kv]
        vc = self._np(self.v_cache_cpu)[self.s0:self.s0 + self.Bk, :, :self.n_kv]
        return oracle.flash_attn_ext(self.q_cpu.numpy(), kc, vc, self._np(self.mask_cpu),
                                     None if self.sinks_cpu is None else self.sinks_cpu.numpy(), scale=scale,
                                     max_bias=max_bias, softcap=softcap, mode=mode, k_type=kt, v_type=kt,
                                     d=self.D, dv=self.D)

    def op(self, scale=None, max_bias=0.0, softcap=0.0):
        return acefa.Op(self.q, self.k, self.v, mask=self.mask, sinks=self.sinks, kv_type=self.kv_type,
                        scale=scale, max_bias=max_bias, softcap=softcap)

    def gpu(self, **kw):
        o = self.op(**kw)
        out = o()
        torch.cuda.synchronize()
        return out.cpu().numpy()
