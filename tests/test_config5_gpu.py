"""GPU parity of the attention shapes of BASELINE config 5 (one generation of
the Qwen3-4B LM over a Q8_0 KV cache) against the CPU oracle, through the C
ABI, at the north-star tolerance (max-abs 2e-3, cosine >= 0.99995).

* the 512-token prompt prefill of one KV set (qw3lm_forward,
  src/qwen3-lm.h:480-621): Q [128, 512, 32], K/V views [128, 512, 8] of set s
  of a [128, max_seq, 8, 16] cache, causal mask [512, 512];
* batched decode steps (qw3lm_forward_batch, src/qwen3-lm.h:629-894) at the
  first and last windows of the generation, n_kv_pad = PAD(kv_len, 256) = 768
  and 2560 (src/qwen3-lm.h:496-500), with each set's valid length inside the
  window (mask [n_kv_pad, 1, 1, 16]: 0 before kv_len, -inf after);
* the same steps over an F16 cache (the reference's own cache type,
  src/qwen3-lm.h:228-229).
"""
import numpy as np
import pytest

import acefa
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu

MAX_SEQ = 2560  # PAD(512 + 2000, 256)


@pytest.mark.parametrize("kv", ["q8_0", "f16"])
def test_prompt_prefill_512_over_cache(kv):
    c = Case(42 + 5000 + 1, B=1, Hq=32, Hkv=8, n_q=512, n_kv=512, kv=kv, max_seq=MAX_SEQ, s0=3, mask="causal")
    got = c.gpu()
    assert_close(got, c.oracle(), what=f"prefill 512 {kv}")
    assert acefa.device_error() == 0


@pytest.mark.parametrize("kv", ["q8_0", "f16"])
@pytest.mark.parametrize("window,first_len", [(768, 513), (2560, 2305)])
def test_decode_step_window(kv, window, first_len):
    """16 sets (8 requests x CFG); valid lengths spread over the window, the
    cond / uncond pair of a request differing by a few tokens."""
    valid = [min(window, first_len + 13 * (i // 2) + 3 * (i % 2)) for i in range(16)]
    c = Case(42 + 5000 + window + first_len, B=16, Hq=32, Hkv=8, n_q=1, n_kv=window, kv=kv, max_seq=MAX_SEQ,
             mask="valid", valid=valid)
    got = c.gpu()
    assert acefa.last_path() == 1 and acefa.last_launch_count() == 1
    assert_close(got, c.oracle(), what=f"decode window {window} {kv}")
    assert acefa.device_error() == 0


def test_decode_window_tail_garbage_is_ignored():
    """Cache rows past each set's kv_len hold stale values of a previous
    generation; the -inf mask must remove them exactly (Q8_0 blocks with large
    scales)."""
    valid = [513 + 17 * i for i in range(16)]
    c = Case(42 + 5000 + 77, B=16, Hq=32, Hkv=8, n_q=1, n_kv=768, kv="q8_0", max_seq=MAX_SEQ, mask="valid",
             valid=valid)
    kf = np.random.default_rng(5077).standard_normal((16, 8, MAX_SEQ, 128)).astype(np.float32) * 3000.0
    big = acefa.quantize_q8_0(__import__("torch").from_numpy(kf))
    for s in range(16):
        c.k_cache_cpu[s, :, valid[s]:] = big[s, :, valid[s]:]
        c.v_cache_cpu[s, :, valid[s]:] = big[s, :, valid[s]:]
    c.to("cuda")
    assert_close(c.gpu(), c.oracle(), what="stale tail")
