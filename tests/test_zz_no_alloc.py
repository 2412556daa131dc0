"""acefa_flash_attn_ext_noalloc: the operator for callers that cannot give the
engine any device memory (a host whose allocator owns every buffer, a thread
that must not block on cudaMalloc, a build that forbids runtime allocation).

Its scratch (the dense path's mask-class table and split partials) is a fixed
array inside the library, so these tests check
that it produces the same result as the allocating entry point, call after
call, and that it refuses operands whose scratch would not fit.  This file is
collected last so that a stopping run has already exercised everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

import acefa
import oracle
from fa_cases import Case, assert_close

NOALLOC_BYTES = 8 << 20  # the fixed array's size, as include/acefa.h states it

pytestmark = pytest.mark.gpu


def _noalloc(op, stream=None):
    lib = acefa.load_library()
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    s = torch.cuda.current_stream() if stream is None else stream
    return lib.acefa_flash_attn_ext_noalloc(r(op.tq), r(op.tk), r(op.tv), r(op.tm), r(op.ts), r(op.td), op.scale,
                                            op.max_bias, op.softcap, op.prec, ctypes.c_void_p(s.cuda_stream))


@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_noalloc_matches_allocating_entry_twice(kv):
    # two different operand sets back to back: the second call finds the first
    # call's leftovers in the shared scratch and must not be affected by them
    cases = [
        Case(4242, B=16, Hq=32, Hkv=8, n_q=1, n_kv=2048, kv=kv, max_seq=4096, mask="valid",
             valid=[2048 - 37 * i for i in range(16)]),
        Case(4243, B=4, Hq=16, Hkv=8, n_q=3, n_kv=777, kv=kv, mask="random", sinks=True),
    ]
    for c in cases:
        ref_op = c.op()
        want = ref_op().clone()
        torch.cuda.synchronize()
        op = c.op()  # separate output buffer for the no-alloc call
        op.out.fill_(float("nan"))
        st = _noalloc(op)
        assert st == 0, acefa.STATUS_NAMES.get(st, st)
        torch.cuda.synchronize()
        assert_close(op.out.cpu().numpy(), want.cpu().numpy(), what=f"noalloc {kv}")
        assert acefa.device_error() == 0


def _oracle_rows(c, rows):
    q = np.ascontiguousarray(c.q_cpu.numpy()[:, :, rows])
    kc = c.k_cache_cpu.numpy()[:, :, :c.n_kv]
    vc = c.v_cache_cpu.numpy()[:, :, :c.n_kv]
    m = None if c.mask_cpu is None else np.ascontiguousarray(c.mask_cpu.numpy()[:, :, rows])
    return oracle.flash_attn_ext(q, kc, vc, m, scale=c.D ** -0.5, k_type=oracle.GGML_F16, v_type=oracle.GGML_F16,
                                 d=c.D, dv=c.D)


def test_noalloc_dense_runs_within_the_fixed_array():
    """Dense (tcgen05) operands whose preferred last-wave split would need more
    scratch than the fixed array holds: 512 work units on 148 SMs leave 68 in
    the last wave, and splitting them would take ~18 MB of partials.  Given
    8 MiB, the plan drops the split instead of refusing the call.  The result
    must equal, bit for bit, the allocating entry given an 8 MiB workspace
    (the same plan), and meet the oracle on sampled rows -- on a second call
    too, after a decode call and a masked dense call have left their own data
    in the shared array."""
    rows = [0, 1, 127, 128, 2047, 4095]
    big = Case(4244, B=1, Hq=32, Hkv=8, n_q=4096, n_kv=4096, mask=None)
    # a decode call and a masked dense call (class table in the array) between the two dense runs
    dec = Case(4245, B=8, Hq=32, Hkv=8, n_q=1, n_kv=1536, mask="valid", valid=[1536 - 100 * i for i in range(8)])
    msk = Case(4246, B=2, Hq=16, Hkv=8, n_q=700, n_kv=900, mask="random", m_batch=1)
    ref_big = big.op()
    ref_big.workspace = torch.empty(NOALLOC_BYTES, dtype=torch.uint8, device="cuda")
    want_big = ref_big().clone()
    assert acefa.last_path() == 2
    want_msk = msk.op()().clone()
    want_dec = dec.op()().clone()
    torch.cuda.synchronize()
    for rep in range(2):
        for c, want in ((big, want_big), (dec, want_dec), (msk, want_msk)):
            op = c.op()
            op.out.fill_(float("nan"))
            st = _noalloc(op)
            assert st == 0, acefa.STATUS_NAMES.get(st, st)
            torch.cuda.synchronize()
            got = op.out.cpu().numpy()
            if c is big:
                assert np.array_equal(got, want.cpu().numpy()), f"dense no-alloc call {rep} differs"
                assert_close(got[:, rows], _oracle_rows(c, rows), what=f"dense noalloc rows, call {rep}")
            else:
                assert_close(got, want.cpu().numpy(), what=f"noalloc call {rep}")
    assert_close(want_msk.cpu().numpy(), msk.oracle(), what="masked dense vs oracle")
    assert acefa.device_error() == 0


def test_noalloc_refuses_oversized_operands():
    # A masked dense node whose mask-class table alone (one byte per mask batch
    # x 128-row tile x 128-key tile: 160 x 128 x 512 = 10 MiB) exceeds the fixed
    # 8 MiB; descriptors only (nothing is launched, so no memory behind them)
    lib = acefa.load_library()
    D, Hq, Hkv, B, nkv, nq = 128, 8, 8, 160, 65536, 16384

    def td(ne, es, gtype):
        t = acefa.Tensor()
        t.type = gtype
        t.ne[:] = ne
        nb = [es]
        for i in range(1, 4):
            nb.append(nb[-1] * ne[i - 1])
        t.nb[:] = nb
        t.data = 1 << 20
        return t

    q = td([D, nq, Hq, B], 4, acefa.GGML_F32)
    k = td([D, nkv, Hkv, B], 2, acefa.GGML_F16)
    v = td([D, nkv, Hkv, B], 2, acefa.GGML_F16)
    m = td([nkv, nq, 1, B], 2, acefa.GGML_F16)
    d = td([D, Hq, nq, B], 4, acefa.GGML_F32)
    r = ctypes.byref
    assert lib.acefa_workspace_bytes(r(q), r(k), r(v), r(m), r(d)) > (8 << 20)
    st = lib.acefa_flash_attn_ext_noalloc(r(q), r(k), r(v), r(m), None, r(d), 0.088, 0.0, 0.0, 10, None)
    assert st == -9
    assert b"no-alloc" in lib.acefa_status_string(st)
