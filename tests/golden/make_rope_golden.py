"""Golden vectors of the attention prologue (QK-norm + RoPE NEOX), generated
with the Qwen3 model definition of HF transformers (Qwen3RMSNorm,
Qwen3RotaryEmbedding, apply_rotary_pos_emb: the upstream modules whose
weights acestep.cpp's GGUFs carry; ggml's own rope kernel lives in the absent
ggml submodule).  Test infrastructure: tests/test_oracle.py checks the
oracle's ora_rope_norm against these.

Run from the repository root (needs transformers, CPU only):
    python tests/golden/make_rope_golden.py
"""
import os

import numpy as np
import torch
from transformers import Qwen3Config
from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, Qwen3RotaryEmbedding, apply_rotary_pos_emb

HERE = os.path.dirname(os.path.abspath(__file__))


def make(name, D, theta, eps, positions, seed):
    g = torch.Generator().manual_seed(seed)
    rows = len(positions)
    x = torch.randn(rows, D, generator=g) * 3.0
    w = 1.0 + 0.25 * torch.randn(D, generator=g)
    cfg = Qwen3Config(head_dim=D, hidden_size=D * 4, num_attention_heads=4, num_key_value_heads=4,
                      rms_norm_eps=eps, rope_parameters={"rope_type": "default", "rope_theta": theta},
                      max_position_embeddings=1 << 16)
    norm = Qwen3RMSNorm(D, eps=eps)
    with torch.no_grad():
        norm.weight.copy_(w)
        y = norm(x)
    rot = Qwen3RotaryEmbedding(cfg)
    pos = torch.tensor(positions, dtype=torch.int64).view(1, rows)
    cos, sin = rot(y.view(1, rows, D), pos)
    # apply_rotary_pos_emb takes (batch, heads, seq, D)
    q = y.view(1, 1, rows, D)
    qr, _ = apply_rotary_pos_emb(q, q, cos, sin)
    np.savez(os.path.join(HERE, f"rope_norm_{name}.npz"), x=x.numpy(), weight=w.numpy(),
             positions=np.array(positions, dtype=np.int32), eps=np.float32(eps), theta=np.float32(theta),
             normed=y.numpy(), out=qr.view(rows, D).numpy())


if __name__ == "__main__":
    # Qwen3 LM / DiT / encoders: head_dim 128, rope_theta 1e6, rms_norm_eps 1e-6
    # (src/qwen3-lm.h:172-173, src/cond-enc.h:26-27); small, mid and long positions
    make("d128", 128, 1.0e6, 1e-6, [0, 1, 2, 3, 17, 63, 64, 255, 1000, 4095, 6000, 8191], seed=11)
    make("d64", 64, 1.0e4, 1e-5, [0, 1, 5, 31, 500, 2047], seed=12)
