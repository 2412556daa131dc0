"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and validates operands exactly like the ggml operator contract."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

import acefa

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "acefa.h")


@pytest.fixture(scope="module")
def lib():
    import importlib.util

    spec = importlib.util.spec_from_file_location("acestep_build", os.path.join(ROOT, "acestep.cpp_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    return acefa.load_library()


def header_functions():
    txt = open(HEADER).read()
    return re.findall(r"ACEFA_API\s+[\w\s\*]+?\b(acefa_\w+)\s*\(", txt)


def test_header_declares_expected_api():
    names = header_functions()
    assert set(names) == set(acefa.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.check_output(["nm", "-D", "--defined-only", acefa.LIB_PATH], text=True)
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in header_functions():
        assert name in exported, name
        assert hasattr(lib, name)
    # nothing else leaks out of the library's C++ internals
    leaked = [s for s in exported if s.startswith("_ZN5acefa")]
    assert not leaked, leaked[:5]


def test_status_strings(lib):
    for code in range(-8, 1):
        s = lib.acefa_status_string(code)
        assert s and s != b"unknown status"
    assert lib.acefa_version() >= 100


def _td(shape_ne, nb, gtype, ptr=256):
    t = acefa.Tensor()
    t.type = gtype
    t.ne[:] = shape_ne
    t.nb[:] = nb
    t.data = ptr
    return t


def _contig(ne, es):
    nb = [es]
    for i in range(1, 4):
        nb.append(nb[-1] * ne[i - 1])
    return nb


def _ops(D=128, nq=1, Hq=16, B=1, nkv=2048, Hkv=8, Bk=1, kt=acefa.GGML_F16, mask=True):
    q = _td([D, nq, Hq, B], _contig([D, nq, Hq, B], 4), acefa.GGML_F32)
    if kt == acefa.GGML_Q8_0:
        knb = [34, D // 32 * 34, D // 32 * 34 * nkv, D // 32 * 34 * nkv * Hkv]
    else:
        knb = _contig([D, nkv, Hkv, Bk], 2)
    k = _td([D, nkv, Hkv, Bk], knb, kt)
    v = _td([D, nkv, Hkv, Bk], knb, kt)
    m = _td([nkv, nq, 1, B], _contig([nkv, nq, 1, B], 2), acefa.GGML_F16) if mask else None
    d = _td([D, Hq, nq, B], _contig([D, Hq, nq, B], 4), acefa.GGML_F32)
    return q, k, v, m, d


def _check(lib, q, k, v, m, d, s=None):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    return lib.acefa_check(r(q), r(k), r(v), r(m), r(s), r(d))


def test_check_accepts_reference_shapes(lib):
    # config 1 (Qwen3-0.6B decode), config 2 (4B batched decode), DiT self/cross
    assert _check(lib, *_ops()) == 0
    assert _check(lib, *_ops(Hq=32, B=16, Bk=16, nkv=8192)) == 0
    assert _check(lib, *_ops(Hq=32, B=16, Bk=16, nkv=8192, kt=acefa.GGML_Q8_0)) == 0
    assert _check(lib, *_ops(nq=1500, Hq=16, Hkv=16, B=2, Bk=2, nkv=1500, mask=False)) == 0
    assert _check(lib, *_ops(nq=6000, Hq=16, Hkv=16, B=2, Bk=2, nkv=512)) == 0
    assert _check(lib, *_ops(D=64, kt=acefa.GGML_BF16)) == 0
    assert _check(lib, *_ops(D=256)) == 0                      # D = 256: F16 and BF16 K/V
    assert _check(lib, *_ops(D=256, kt=acefa.GGML_BF16)) == 0
    assert _check(lib, *_ops(D=256, kt=acefa.GGML_Q8_0)) == -2


def test_check_rejects_contract_violations(lib):
    q, k, v, m, d = _ops()
    assert _check(lib, None, k, v, m, d) == -1
    bad = _ops(Hq=12, Hkv=8)  # 12 % 8 != 0
    assert _check(lib, *bad) == -3
    q2, k2, v2, m2, d2 = _ops()
    q2.type = acefa.GGML_F16
    assert _check(lib, q2, k2, v2, m2, d2) == -2
    q3, k3, v3, m3, d3 = _ops()
    v3.type = acefa.GGML_BF16  # K and V types differ
    assert _check(lib, q3, k3, v3, m3, d3) == -2
    q4, k4, v4, m4, d4 = _ops()
    m4.ne[0] = 100  # mask narrower than n_kv
    assert _check(lib, q4, k4, v4, m4, d4) == -3
    q5, k5, v5, m5, d5 = _ops(D=96)
    assert _check(lib, q5, k5, v5, m5, d5) == -3
    q6, k6, v6, m6, d6 = _ops()
    k6.nb[1] = 264  # row stride not 16-B aligned
    assert _check(lib, q6, k6, v6, m6, d6) == -4
    q7, k7, v7, m7, d7 = _ops()
    k7.data = 256 + 8  # K base not 16-B aligned
    assert _check(lib, q7, k7, v7, m7, d7) == -4
    q8, k8, v8, m8, d8 = _ops()
    d8.ne[1] = 8  # dst not [D, Hq, n_q, B]
    assert _check(lib, q8, k8, v8, m8, d8) == -3
    q9, k9, v9, m9, d9 = _ops(kt=acefa.GGML_Q8_0)
    k9.nb[1] = 144  # Q8_0 rows must be contiguous blocks
    assert _check(lib, q9, k9, v9, m9, d9) == -4


def test_supports_mirrors_check(lib):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    ok = _ops()
    assert lib.acefa_supports(*[r(x) for x in ok[:4]], None, r(ok[4])) == 1
    bad = _ops(Hq=12)
    assert lib.acefa_supports(*[r(x) for x in bad[:4]], None, r(bad[4])) == 0


def test_flash_attn_without_gpu_fails_cleanly(lib):
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    q, k, v, m, d = _ops()
    st = lib.acefa_flash_attn_ext(r(q), r(k), r(v), r(m), None, r(d), 0.088, 0.0, 0.0, 10, None, None, 0)
    assert st in (-6, -7)  # CUDA error / not an sm_100 device: no launch, no crash
    assert lib.acefa_workspace_bytes(r(q), r(k), r(v), r(m), r(d)) == 0


def test_mirrored_entry_validates_mirrors_before_launch(lib):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    q, k, v, m, d = _ops()
    d.data = 4096

    def call(ptrs, n):
        arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs) if ptrs is not None else None
        return lib.acefa_flash_attn_ext_mirrored(r(q), r(k), r(v), r(m), None, r(d), 0.088, 0.0, 0.0, 10,
                                                 arr, n, None, None, 0)

    assert call(None, 1) == -1                   # mirrors NULL
    assert call([0], 1) == -1                    # a NULL mirror
    assert call([(1 << 30) + 4100], 1) == -4  # not congruent to dst mod 16
    assert call([4096], 1) == -4                 # the mirror is dst itself
    assert call([1 << 30] * 8, 8) == -3          # more than ACEFA_MAX_MIRRORS
    assert call([1 << 30], -1) == -3
    # valid mirrors pass validation and fail only at the device step here
    if not torch.cuda.is_available():
        assert call([(1 << 30) + 4096, (1 << 31) + 4096], 2) in (-6, -7)


def test_append_entry_validates_before_launch(lib):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    q, k, v, m, d = _ops(Hq=32, B=4, Bk=4, nkv=700)
    kn = _td([128, 1, 8, 4], _contig([128, 1, 8, 4], 4), acefa.GGML_F32, ptr=8192)
    vn = _td([128, 1, 8, 4], _contig([128, 1, 8, 4], 4), acefa.GGML_F32, ptr=16384)

    def call(kn_, vn_, pos):
        return lib.acefa_flash_attn_ext_append(r(q), r(k), r(v), r(m), None, r(d), 0.088, 0.0, 0.0, 10,
                                               r(kn_), r(vn_), pos, None, None, 0)

    assert call(kn, vn, None) == -1                   # no positions
    assert call(None, vn, 4096) == -1                 # no new K row
    bad_t = _td([128, 1, 8, 4], _contig([128, 1, 8, 4], 2), acefa.GGML_F16, ptr=8192)
    assert call(bad_t, vn, 4096) == -2                # new rows are f32
    bad_s = _td([128, 2, 8, 4], _contig([128, 2, 8, 4], 4), acefa.GGML_F32, ptr=8192)
    assert call(bad_s, vn, 4096) == -3                # one row per (head, set)
    q2, k2, v2, m2, d2 = _ops(D=256, Hq=32, B=4, Bk=4, nkv=700)
    kn2 = _td([256, 1, 8, 4], _contig([256, 1, 8, 4], 4), acefa.GGML_F32, ptr=8192)
    assert lib.acefa_flash_attn_ext_append(r(q2), r(k2), r(v2), r(m2), None, r(d2), 0.06, 0.0, 0.0, 10, r(kn2),
                                           r(kn2), 4096, None, None, 0) == -3  # D = 256: no fused append
    if not torch.cuda.is_available():
        assert call(kn, vn, 4096) in (-6, -7)         # valid: fails only at the device step


def test_mask_rule_entry_validates_before_launch(lib):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    q, k, v, m, d = _ops(Hq=32, B=4, Bk=4, nkv=700)

    def call(mg):
        return lib.acefa_flash_attn_ext_gen(r(q), r(k), r(v), r(mg), None, r(d), 0.088, 0.0, 0.0, 10, None, None, 0)

    assert call(None) == -1                                                # no rule
    assert call(acefa.mask_gen(0)) == -3                                   # unknown kind
    assert call(acefa.mask_gen(acefa.MASK_WINDOW, window=-1)) == -3        # negative window
    q40, k40, v40, m40, d40 = _ops(Hq=32, B=40, Bk=40, nkv=700)
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[5] * 32)
    assert lib.acefa_flash_attn_ext_gen(r(q40), r(k40), r(v40), r(mg), None, r(d40), 0.088, 0.0, 0.0, 10,
                                        None, None, 0) == -3               # per-batch rule past 32 sets
    if not torch.cuda.is_available():
        assert call(mg) in (-6, -7)                                        # valid: fails only at the device step
        w = acefa.mask_gen(acefa.MASK_WINDOW, window=4)
        assert lib.acefa_flash_attn_ext_gen(r(q40), r(k40), r(v40), r(w), None, r(d40), 0.088, 0.0, 0.0, 10,
                                            None, None, 0) in (-6, -7)     # window: any batch count


def test_fused_entry_validates_before_launch(lib):
    """acefa_flash_attn_ext_fused: every fusion's operands are checked before
    any device work (fake device pointers; nothing may be dereferenced)."""
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    q, k, v, m, d = _ops(Hq=32, B=4, Bk=4, nkv=700)

    def call(ext, mask=m):
        return lib.acefa_flash_attn_ext_fused(r(q), r(k), r(v), r(mask), None, r(d), 0.088, 0.0, 0.0, 10,
                                              r(ext), None, None, 0)

    ext = acefa.OpExt()
    pro = acefa.RopeNormC(4096, 1e-6, 1.0e6, None)
    ext.q_prologue = ctypes.addressof(pro)
    assert call(ext) == -1                                   # RoPE without positions
    bad = acefa.RopeNormC(4096, -1.0, 1.0e6, 8192)
    ext.q_prologue = ctypes.addressof(bad)
    assert call(ext) == -3                                   # negative eps
    odd = acefa.RopeNormC(4098, 1e-6, 0.0, None)
    ext.q_prologue = ctypes.addressof(odd)
    assert call(ext) == -4                                   # misaligned weight
    ext = acefa.OpExt()
    ok = acefa.RopeNormC(4096, 1e-6, 1.0e6, 8192)
    ext.k_prologue = ctypes.addressof(ok)
    assert call(ext) == -3                                   # K prologue without an append
    ext = acefa.OpExt()
    mg = acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[1, 2, 3, 4])
    ext.mask_gen = ctypes.addressof(mg)
    assert call(ext) == -3                                   # rule and mask tensor together
    if not torch.cuda.is_available():
        assert call(ext, mask=None) in (-6, -7)             # valid: fails only at the device step
        ext = acefa.OpExt()
        ext.q_prologue = ctypes.addressof(ok)
        assert call(ext) in (-6, -7)
        assert call(None) in (-6, -7)                        # no options = the plain operator


def test_kv_prologue_validates_before_launch(lib):
    r = lambda x: ctypes.byref(x) if x is not None else None  # noqa: E731
    ne = [128, 300, 8, 2]
    src = _td(ne, _contig(ne, 4), acefa.GGML_F32, ptr=1 << 20)
    dst = _td(ne, _contig(ne, 2), acefa.GGML_F16, ptr=1 << 22)
    pro = acefa.RopeNormC(4096, 1e-6, 1.0e6, 8192)
    assert lib.acefa_kv_prologue(None, None, r(dst), None, r(pro), None) == -1
    assert lib.acefa_kv_prologue(r(src), r(src), r(dst), None, r(pro), None) == -1   # V without a destination
    q8 = _td(ne, _contig(ne, 2), acefa.GGML_Q8_0, ptr=1 << 22)
    assert lib.acefa_kv_prologue(r(src), None, r(q8), None, r(pro), None) == -2     # F16 / BF16 only
    ne2 = [128, 301, 8, 2]
    dst2 = _td(ne2, _contig(ne2, 2), acefa.GGML_F16, ptr=1 << 22)
    assert lib.acefa_kv_prologue(r(src), None, r(dst2), None, r(pro), None) == -3    # shapes differ
    ne96 = [96, 300, 8, 2]
    s96 = _td(ne96, _contig(ne96, 4), acefa.GGML_F32, ptr=1 << 20)
    d96 = _td(ne96, _contig(ne96, 2), acefa.GGML_F16, ptr=1 << 22)
    assert lib.acefa_kv_prologue(r(s96), None, r(d96), None, r(pro), None) == -3     # D 64 or 128
    strided = _td(ne, [8] + _contig(ne, 4)[1:], acefa.GGML_F32, ptr=1 << 20)
    assert lib.acefa_kv_prologue(r(strided), None, r(dst), None, r(pro), None) == -4  # rows contiguous
    if not torch.cuda.is_available():
        assert lib.acefa_kv_prologue(r(src), r(src), r(dst), r(dst), r(pro), None) in (-6, -7)
        assert lib.acefa_kv_prologue(r(src), None, r(dst), None, None, None) in (-6, -7)  # plain conversion


def test_cfg_combine_validates_before_launch(lib):
    f = lib.acefa_cfg_logit_combine
    P = ctypes.c_void_p
    c, u, o = P(1 << 20), P((1 << 20) + 8 * 65559 * 4), P(1 << 26)
    assert f(None, u, 65559, 8, 0, 24, 65535, 2.0, o, None) == -1
    if not torch.cuda.is_available():
        assert f(None, None, 65559, 0, 0, 24, 65535, 2.0, None, None) in (-6, -7)  # n == 0: no buffers needed
    assert f(c, u, 65559, 8, 0, 24, 65535, 2.0, None, None) == -1
    assert f(c, u, 65559, 8, 0, 25, 65535, 2.0, o, None) == -3          # code range past the row
    assert f(c, u, 65559, 8, 65559, 24, 65535, 2.0, o, None) == -3      # EOS column past the row
    assert f(c, u, 65559, -1, 0, 24, 65535, 2.0, o, None) == -3
    assert f(c, u, 65559, 65536, 0, 24, 65535, 2.0, o, None) == -3      # one grid row per sequence
    assert f(c, u, 0, 8, -1, 0, 0, 2.0, o, None) == -3
    assert f(P((1 << 20) + 2), u, 65559, 8, 0, 24, 65535, 2.0, o, None) == -4  # f32 alignment
    assert f(c, u, 65559, 8, 0, 24, 65535, 2.0, P((1 << 20) + 64), None) == -4  # compact overlaps cond
    assert f(c, u, 65559, 8, 0, 24, 65535, 2.0, P((1 << 20) + 9 * 65559 * 4), None) == -4  # ... uncond
    if not torch.cuda.is_available():
        assert f(c, u, 65559, 8, 0, 24, 65535, 2.0, o, None) in (-6, -7)
        assert f(c, u, 100, 8, -1, 0, 100, 2.0, c, None) in (-6, -7)  # in place, full rows: accepted


def test_peer_entry_points_reject_null(lib):
    assert lib.acefa_peer_export(None, None, None) == -1
    assert lib.acefa_peer_import(None, 0, None) == -1
    assert lib.acefa_peer_release(None) == -1
    assert lib.acefa_peer_release(ctypes.c_void_p(4096)) == -1  # never imported


def test_torch_q8_0_quantiser_bit_exact(oracle_mod):
    x = np.load(os.path.join(ROOT, "tests", "golden", "q8_0_input.npy"))
    want = np.load(os.path.join(ROOT, "tests", "golden", "q8_0_gguf.npy"))
    got = acefa.quantize_q8_0(torch.from_numpy(x)).numpy()
    assert np.array_equal(got, want)
    back = acefa.dequantize_q8_0(torch.from_numpy(want)).numpy()
    assert np.array_equal(back, oracle_mod.dequantize_q8_0(want))
