"""acefa_flash_attn_ext_mirrored on one GPU: the mirrors are other buffers of
this device laid out like dst.  Every kernel family's output stage (decode
direct write, split-KV combine, dense tcgen05) must store the identical rows to
dst and to every mirror (bit for bit: the same value goes to every address),
and dst must meet the parity tolerance like the unmirrored call."""
import numpy as np
import pytest
import torch

import acefa
from fa_cases import Case, assert_close

pytestmark = pytest.mark.gpu


def _run_mirrored(case, n_mirrors, **kw):
    out = torch.full((case.B, case.n_q, case.Hq, case.D), float("nan"), device="cuda")
    mirrors = [torch.full_like(out, float("nan")) for _ in range(n_mirrors)]
    op = acefa.Op(case.q, case.k, case.v, mask=case.mask, sinks=case.sinks, kv_type=case.kv_type, out=out,
                  mirrors=[m.data_ptr() for m in mirrors], **kw)
    op()
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for m in mirrors:
        assert (m.cpu().numpy() == got).all()
    return got


@pytest.mark.parametrize("n_kv,B", [(200, 4), (6000, 2)])  # direct write / split-KV + combine
def test_mirrored_decode(n_kv, B):
    c = Case(31, B=B, Hq=16, Hkv=8, n_q=1, n_kv=n_kv, mask="zeros")
    got = _run_mirrored(c, 3)
    assert_close(got, c.oracle(), what="decode mirrored")


def test_mirrored_dense_max_mirrors():
    c = Case(32, B=1, Hq=8, Hkv=4, n_q=300, n_kv=300, mask="causal")
    got = _run_mirrored(c, acefa.MAX_MIRRORS)
    assert_close(got, c.oracle(), what="dense mirrored")


def test_mirrored_head_slices_assemble_full_output():
    """Two head shards written into their slices of one buffer each, mirrored
    into the other's: both buffers end up holding the full operator."""
    c = Case(33, B=2, Hq=16, Hkv=16, n_q=256, n_kv=256, mask=None)
    full = c.gpu()
    bufs = [torch.full((2, 256, 16, 128), float("nan"), device="cuda") for _ in range(2)]
    for r in range(2):
        hs = slice(8 * r, 8 * r + 8)
        view = bufs[r][:, :, hs, :]
        peer = bufs[1 - r][:, :, hs, :]
        acefa.Op(c.q[:, hs].contiguous(), c.k[:, hs], c.v[:, hs], out=view, mirrors=[peer.data_ptr()])()
    torch.cuda.synchronize()
    for b in bufs:
        assert (b.cpu().numpy() == full).all()


def test_mirrored_dense_split_units():
    """Units split over key ranges: the combine kernel writes the mirrors."""
    c = Case(34, B=1, Hq=10, Hkv=10, n_q=4096, n_kv=4096, mask=None)
    out = torch.full((c.B, c.n_q, c.Hq, c.D), float("nan"), device="cuda")
    mirrors = [torch.full_like(out, float("nan")) for _ in range(2)]
    acefa.Op(c.q, c.k, c.v, out=out, mirrors=[m.data_ptr() for m in mirrors])()
    assert acefa.last_launch_count() == 2  # attention, combine
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    for m in mirrors:
        assert (m.cpu().numpy() == got).all()


@pytest.mark.parametrize("kv", ["bf16", "q8_0"])
def test_mirrored_dense_converted_kv(kv):
    """The dense kernel's output stage with BF16 / Q8_0 K/V (the converter
    warps' instances) writes the mirrors too."""
    c = Case(35, B=2, Hq=16, Hkv=8, n_q=300, n_kv=400, kv=kv, mask="causal")
    got = _run_mirrored(c, 2)
    assert acefa.last_path() == 2
    assert_close(got, c.oracle(), what=f"dense mirrored {kv}")
