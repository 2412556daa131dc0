"""CPU restatement of ggml_flash_attn_ext -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package.  The product library (``libacefa.so``) never
links or calls it; it is the checker, never the thing measured or shipped.

Parity status: the attention arithmetic is *parity unpinned* -- the reference
kernel lives in the absent ggml submodule (acestep.cpp ``.gitmodules:1-3``) and
the reference ships no op-level golden vectors.  The Q8_0 block format is pinned
bit-exactly against gguf 0.19.0 (``tests/golden/q8_0_*.npy``).  The
RMSNorm + RoPE prologue (``rope_norm``) is pinned against the Qwen3 model
definition in HF transformers (``tests/golden/rope_norm_*.npz``).  The CFG
logit combine (``cfg_logit_combine``) is the reference's own host loop
(src/pipeline-lm.cpp:471-492) in f32 arithmetic, checked against a numpy
restatement of that loop.
"""
from .oracle import (  # noqa: F401
    GGML_F16,
    GGML_F32,
    GGML_Q8_0,
    GGML_BF16,
    MODE_F32,
    MODE_GGML_CPU,
    build,
    flash_attn_ext,
    quantize_q8_0,
    dequantize_q8_0,
    lib_path,
    rope_norm,
    cfg_logit_combine,
)
