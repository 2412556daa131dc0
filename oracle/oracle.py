"""ctypes binding of the C oracle (oracle/fa_oracle.c).  Test infrastructure.

Tensors are numpy arrays in *torch order* (outermost first): a ggml tensor with
ne = [ne0, ne1, ne2, ne3] is the numpy array of shape (ne3, ne2, ne1, ne0).
Q8_0 tensors are uint8 arrays whose last axis holds the 34-byte blocks of a row.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
MODE_F32, MODE_GGML_CPU = 0, 1

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "fa_oracle.c")
_LIB = os.path.join(_HERE, "_build", "libfa_oracle.so")


def lib_path() -> str:
    return _LIB


def build(force: bool = False) -> str:
    """Compile the oracle with gcc + OpenMP into oracle/_build/."""
    os.makedirs(os.path.dirname(_LIB), exist_ok=True)
    if not force and os.path.exists(_LIB) and os.path.getmtime(_LIB) >= max(
        os.path.getmtime(_SRC), os.path.getmtime(os.path.join(_HERE, "fa_oracle.h"))
    ):
        return _LIB
    cmd = ["gcc", "-O3", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-o", _LIB, _SRC, "-lm"]
    subprocess.check_call(cmd)
    return _LIB


class _Tensor(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("nb", ctypes.c_size_t * 4),
        ("data", ctypes.c_void_p),
    ]


_lib = None


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB)
        P = ctypes.POINTER(_Tensor)
        lib.ora_flash_attn_ext.argtypes = [
            P, P, P, P, P, ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t),
            ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int,
        ]
        lib.ora_flash_attn_ext.restype = ctypes.c_int
        lib.ora_quantize_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.ora_dequantize_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.ora_rope_norm.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_float, ctypes.c_float, ctypes.c_void_p]
        lib.ora_rope_norm.restype = None
        lib.ora_cfg_logit_combine.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                              ctypes.c_void_p]
        lib.ora_cfg_logit_combine.restype = None
        _lib = lib
    return _lib


def _as_tensor(arr: np.ndarray | None, gtype: int, ne0: int | None = None):
    if arr is None:
        return None
    assert arr.ndim == 4
    t = _Tensor()
    t.type = gtype
    shape = list(arr.shape[::-1])
    strides = list(arr.strides[::-1])
    if gtype == GGML_Q8_0:
        assert arr.dtype == np.uint8 and ne0 is not None
        assert strides[0] == 1, "Q8_0 rows must be contiguous blocks"
        shape[0] = ne0
        strides[0] = 34
    t.ne[:] = shape
    t.nb[:] = strides
    t.data = arr.ctypes.data
    return t


def flash_attn_ext(q, k, v, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0,
                   mode=MODE_F32, k_type=None, v_type=None, d=None, dv=None, nthreads=0):
    """Run the oracle.  q: f32 (B, Hq, n_q, D); k/v: f16/bf16(uint16)/f32 arrays
    (Bk, Hkv, n_kv, D) or Q8_0 bytes; mask: f16 (Bm, Hm, >=n_q, n_kv) or None.
    Returns f32 (B, n_q, Hq, Dv) == ggml dst [Dv, Hq, n_q, B]."""
    lib = _load()

    def ty(a, t):
        if t is not None:
            return t
        if a.dtype == np.float32:
            return GGML_F32
        if a.dtype == np.float16:
            return GGML_F16
        raise ValueError("pass k_type/v_type for bf16/q8_0 arrays")

    kt, vt = ty(k, k_type), ty(v, v_type)
    D = q.shape[-1]
    Dv = dv if dv is not None else (v.shape[-1] if vt != GGML_Q8_0 else v.shape[-1] // 34 * 32)
    B, Hq, n_q = q.shape[0], q.shape[1], q.shape[2]
    out = np.zeros((B, n_q, Hq, Dv), dtype=np.float32)
    tq = _as_tensor(q, GGML_F32)
    tk = _as_tensor(k, kt, D)
    tv = _as_tensor(v, vt, Dv)
    tm = _as_tensor(mask, GGML_F16) if mask is not None else None
    ts = None
    if sinks is not None:
        s4 = np.ascontiguousarray(sinks, dtype=np.float32).reshape(1, 1, 1, -1)
        ts = _as_tensor(s4, GGML_F32)
    nb = (ctypes.c_size_t * 4)(*out.strides[::-1])
    rc = lib.ora_flash_attn_ext(
        ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
        ctypes.byref(tm) if tm is not None else None,
        ctypes.byref(ts) if ts is not None else None,
        out.ctypes.data, nb, scale, max_bias, softcap, mode, nthreads,
    )
    if rc != 0:
        raise ValueError(f"oracle rejected the operands (status {rc})")
    return out


def rope_norm(x: np.ndarray, weight=None, eps=1e-6, theta=0.0, positions=None) -> np.ndarray:
    """RMSNorm (times weight) + RoPE NEOX over the last axis (D).  positions
    holds one int per row of x.reshape(-1, D).  Returns a new f32 array."""
    lib = _load()
    y = np.array(x, dtype=np.float32, order="C", copy=True)
    D = y.shape[-1]
    rows = y.size // D
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    p = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32).reshape(-1)
    if theta > 0.0:
        assert p is not None and p.size == rows
    lib.ora_rope_norm(y.ctypes.data, rows, D, None if w is None else w.ctypes.data, eps, theta,
                      None if p is None else p.ctypes.data)
    return y


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """f32 (..., n) -> uint8 (..., n/32*34) Q8_0 blocks."""
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    assert n % 32 == 0
    y = np.empty(x.shape[:-1] + (n // 32 * 34,), dtype=np.uint8)
    lib.ora_quantize_q8_0(x.ctypes.data, y.ctypes.data, x.size)
    return y


def dequantize_q8_0(y: np.ndarray) -> np.ndarray:
    lib = _load()
    y = np.ascontiguousarray(y, dtype=np.uint8)
    n = y.shape[-1] // 34 * 32
    x = np.empty(y.shape[:-1] + (n,), dtype=np.float32)
    lib.ora_dequantize_q8_0(y.ctypes.data, x.ctypes.data, x.size)
    return x


def cfg_logit_combine(cond: np.ndarray, uncond: np.ndarray | None, eos_idx: int, code_offset: int,
                      code_count: int, cfg_scale: float) -> np.ndarray:
    """CFG combine + compaction of n logit rows (cond / uncond: (n, row_stride)
    f32).  Returns (n, code_count + (eos_idx >= 0)) f32."""
    lib = _load()
    c = np.ascontiguousarray(cond, dtype=np.float32)
    u = None if uncond is None else np.ascontiguousarray(uncond, dtype=np.float32)
    n, stride = c.shape
    if u is not None:
        assert u.shape == c.shape
    cols = code_count + (1 if eos_idx >= 0 else 0)
    assert code_offset >= 0 and code_offset + code_count <= stride and eos_idx < stride
    out = np.empty((n, cols), dtype=np.float32)
    lib.ora_cfg_logit_combine(c.ctypes.data, None if u is None else u.ctypes.data, stride, n, eos_idx,
                              code_offset, code_count, cfg_scale, out.ctypes.data)
    return out
