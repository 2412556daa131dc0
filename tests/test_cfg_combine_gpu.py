"""GPU parity of acefa_cfg_logit_combine (the CFG combine and logit compaction
of a batched LM decode step, src/pipeline-lm.cpp:471-492) against the CPU
oracle: bit-exact, through the C ABI.

Layouts of the reference: the partial LM head (out_V = V - TOKEN_IM_END =
65559, EOS at column 0, codes from column AUDIO_CODE_BASE - TOKEN_IM_END = 24)
and the full vocabulary (out_V = 217204, EOS 151645, codes from 151669), each
with uncond rows n_active rows after the cond rows of one batch buffer; the
full-row in-place combine of the first-token sampling (:104-108, :364-370).
"""
import numpy as np
import pytest
import torch

import acefa
import oracle

pytestmark = pytest.mark.gpu

TOKEN_IM_END, AUDIO_CODE_BASE, AUDIO_CODE_COUNT, VOCAB = 151645, 151669, 65535, 217204


def _logits(seed, rows, V):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, V, generator=g) * 12.0
    x[0, :7] = torch.tensor([float("inf"), float("-inf"), float("nan"), 3.0e38, -3.0e38, -1.0e9, 0.0])
    if rows > 1:
        x[-1, -5:] = torch.tensor([float("-inf"), float("inf"), -0.0, 1.0e-45, 2.5e38])
    return x


@pytest.mark.parametrize("partial", [True, False])
@pytest.mark.parametrize("n_active", [1, 3, 8])
@pytest.mark.parametrize("cfg_scale", [2.0, 1.7, 0.0])
def test_batch_layout_bit_exact(partial, n_active, cfg_scale):
    out_V = VOCAB - TOKEN_IM_END if partial else VOCAB
    eos = 0 if partial else TOKEN_IM_END
    off = AUDIO_CODE_BASE - TOKEN_IM_END if partial else AUDIO_CODE_BASE
    use_cfg = cfg_scale > 1.0  # the reference's switch (src/pipeline-lm.cpp:279)
    x = _logits(900 + n_active + int(partial), 2 * n_active, out_V)
    dev = x.cuda()
    cond = dev[:n_active]
    unc = dev[n_active:] if use_cfg else None
    got = acefa.cfg_logit_combine(cond, unc, eos, off, AUDIO_CODE_COUNT, cfg_scale)
    assert acefa.last_launch_count() == 1
    xn = x.numpy()
    want = oracle.cfg_logit_combine(xn[:n_active], xn[n_active:] if use_cfg else None, eos, off,
                                    AUDIO_CODE_COUNT, cfg_scale)
    assert got.shape == (n_active, AUDIO_CODE_COUNT + 1)
    g = got.cpu().numpy()
    assert np.array_equal(g.view(np.uint32)[~np.isnan(want)], want.view(np.uint32)[~np.isnan(want)])
    assert np.array_equal(np.isnan(g), np.isnan(want))


def test_full_row_in_place():
    """lg[v] = lu[v] + cfg_scale * (lg[v] - lu[v]) over the whole row, written
    over the cond rows."""
    n, V = 4, VOCAB
    x = _logits(77, 2 * n, V)
    dev = x.cuda()
    cond = dev[:n]
    acefa.cfg_logit_combine(cond, dev[n:], -1, 0, V, 3.0, out=cond)
    xn = x.numpy()
    want = oracle.cfg_logit_combine(xn[:n], xn[n:], -1, 0, V, 3.0)
    g = dev[:n].cpu().numpy()
    ok = ~np.isnan(want)
    assert np.array_equal(g[ok].view(np.uint32), want[ok].view(np.uint32))
    assert np.array_equal(np.isnan(g), np.isnan(want))
    assert torch.equal(dev[n:].cpu(), x[n:])  # uncond rows untouched


def test_strided_rows_and_no_eos():
    """Rows farther apart than the logits they hold (a padded batch buffer);
    no EOS column."""
    n, V, stride = 5, 1000, 1024
    buf = _logits(5, 2 * n, stride)
    dev = buf.cuda()
    cond = dev[:n, :V]
    unc = dev[n:, :V]
    got = acefa.cfg_logit_combine(cond, unc, -1, 100, 777, 2.25)
    bn = buf.numpy()
    want = oracle.cfg_logit_combine(bn[:n, :V], bn[n:, :V], -1, 100, 777, 2.25)
    gn = got.cpu().numpy()
    ok = ~np.isnan(want)
    assert np.array_equal(gn[ok].view(np.uint32), want[ok].view(np.uint32))


def test_zero_sequences_launch_nothing():
    dev = torch.zeros(1, 64, device="cuda")
    out = torch.empty(0, 10, device="cuda")
    acefa.cfg_logit_combine(dev[:0], dev[:0], 0, 1, 9, 2.0, out=out)
    assert acefa.last_launch_count() == 0


def test_captured_in_a_graph():
    n, out_V = 8, VOCAB - TOKEN_IM_END
    x = _logits(31, 2 * n, out_V).cuda()
    out = torch.empty(n, AUDIO_CODE_COUNT + 1, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        acefa.cfg_logit_combine(x[:n], x[n:], 0, 24, AUDIO_CODE_COUNT, 2.0, out=out, stream=s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            acefa.cfg_logit_combine(x[:n], x[n:], 0, 24, AUDIO_CODE_COUNT, 2.0, out=out, stream=s)
    x.copy_(_logits(32, 2 * n, out_V).cuda())
    g.replay()
    torch.cuda.synchronize()
    xn = x.cpu().numpy()
    want = oracle.cfg_logit_combine(xn[:n], xn[n:], 0, 24, AUDIO_CODE_COUNT, 2.0)
    gn = out.cpu().numpy()
    ok = ~np.isnan(want)
    assert np.array_equal(gn[ok].view(np.uint32), want[ok].view(np.uint32))
