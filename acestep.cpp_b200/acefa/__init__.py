"""Python host side of the acefa attention engine (ctypes over include/acefa.h).

The operator is ggml_flash_attn_ext; tensors are torch tensors whose dims are
ggml's ne[] reversed (torch shape (ne3, ne2, ne1, ne0)), so a ggml Q
[D, n_q, Hq, B] is a torch tensor of shape (B, Hq, n_q, D) and the result
[D, Hq, n_q, B] comes back with shape (B, n_q, Hq, D).  Q8_0 K/V are uint8
tensors whose last axis holds a row's 34-byte blocks (D/32 of them).

There is no fallback: if libacefa.so is missing or the current device is not
an sm_100 GPU every call raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
PREC_DEFAULT, PREC_F32 = 0, 10

OK = 0
STATUS_NAMES = {
    0: "ACEFA_OK", -1: "ACEFA_ERR_NULL", -2: "ACEFA_ERR_TYPE", -3: "ACEFA_ERR_SHAPE",
    -4: "ACEFA_ERR_LAYOUT", -5: "ACEFA_ERR_WORKSPACE", -6: "ACEFA_ERR_CUDA",
    -7: "ACEFA_ERR_DEVICE", -8: "ACEFA_ERR_DEVICE_TIMEOUT", -9: "ACEFA_ERR_NOALLOC_LIMIT",
}

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# ACEFA_LIBRARY selects another build of the same ABI (e.g. a variant compiled
# with different tuning macros); by default the in-tree library is used.
LIB_PATH = os.environ.get("ACEFA_LIBRARY") or os.path.join(_PKG_DIR, "libacefa.so")

EXPORTED_SYMBOLS = (
    "acefa_flash_attn_ext",
    "acefa_workspace_bytes",
    "acefa_supports",
    "acefa_check",
    "acefa_device_error",
    "acefa_status_string",
    "acefa_last_launch_count",
    "acefa_last_path",
    "acefa_version",
    "acefa_flash_attn_ext_noalloc",
    "acefa_flash_attn_ext_mirrored",
    "acefa_peer_export",
    "acefa_peer_import",
    "acefa_peer_release",
    "acefa_flash_attn_ext_append",
    "acefa_flash_attn_ext_gen",
    "acefa_flash_attn_ext_fused",
    "acefa_kv_prologue",
    "acefa_cfg_logit_combine",
)

MAX_MIRRORS = 7
PEER_HANDLE_BYTES = 64

# mask rules (acefa_mask_gen)
MASK_CAUSAL, MASK_WINDOW, MASK_PADDING = 1, 2, 3
MASK_GEN_MAX_BATCH = 32


class MaskGen(ctypes.Structure):
    """acefa_mask_gen: a 0 / -inf mask given by its rule."""
    _fields_ = [("kind", ctypes.c_int32), ("window", ctypes.c_int32),
                ("pos0", ctypes.c_int64 * MASK_GEN_MAX_BATCH), ("len", ctypes.c_int64 * MASK_GEN_MAX_BATCH)]


def mask_gen(kind: int, window: int = 0, pos0=(), lens=()) -> MaskGen:
    m = MaskGen()
    m.kind, m.window = int(kind), int(window)
    for i, p in enumerate(pos0):
        m.pos0[i] = int(p)
    for i, n in enumerate(lens):
        m.len[i] = int(n)
    return m


def rule_mask(m: MaskGen, B: int, n_q: int, n_kv: int, ne0: int | None = None, device="cuda") -> torch.Tensor:
    """The f16 mask tensor (B, 1, n_q, ne0) a rule stands for: 0 where key j is
    visible to query i of batch b, -inf elsewhere (and past n_kv)."""
    ne0 = ne0 or n_kv
    j = torch.arange(ne0).view(1, 1, ne0)
    i = torch.arange(n_q).view(1, n_q, 1)
    if m.kind == MASK_CAUSAL:
        vis = j <= torch.tensor([m.pos0[b] for b in range(B)]).view(B, 1, 1) + i
    elif m.kind == MASK_WINDOW:
        vis = (i - j).abs() <= m.window
        vis = vis.expand(B, n_q, ne0)
    else:
        vis = (j < torch.tensor([m.len[b] for b in range(B)]).view(B, 1, 1)).expand(B, n_q, ne0)
    vis = vis & (j < n_kv)
    out = torch.full((B, 1, n_q, ne0), float("-inf"), dtype=torch.float16)
    out[:, 0][vis] = 0.0
    return out.to(device)


class RopeNormC(ctypes.Structure):
    """acefa_rope_norm: RMSNorm (times a weight) + RoPE NEOX of rows of D values."""
    _fields_ = [("norm_weight", ctypes.c_void_p), ("eps", ctypes.c_float), ("theta_base", ctypes.c_float),
                ("positions", ctypes.c_void_p)]


class RopeNorm:
    """A prologue description that keeps its device tensors alive.
    weight: (D,) f32 CUDA tensor or None; positions: int32 CUDA tensor or None."""

    def __init__(self, weight=None, eps=1e-6, theta=0.0, positions=None):
        if positions is not None and (positions.dtype != torch.int32 or not positions.is_cuda):
            raise ValueError("positions: int32 CUDA tensor (ggml's positions)")
        if weight is not None and (weight.dtype != torch.float32 or not weight.is_cuda or not weight.is_contiguous()):
            raise ValueError("weight: contiguous f32 CUDA tensor")
        self.weight, self.positions = weight, positions
        self.eps, self.theta = float(eps), float(theta)
        self.c = RopeNormC(weight.data_ptr() if weight is not None else None, self.eps, self.theta,
                           positions.data_ptr() if positions is not None else None)


class OpExt(ctypes.Structure):
    """acefa_op_ext."""
    _fields_ = [("mask_gen", ctypes.c_void_p), ("q_prologue", ctypes.c_void_p), ("k_new", ctypes.c_void_p),
                ("v_new", ctypes.c_void_p), ("append_pos", ctypes.c_void_p), ("k_prologue", ctypes.c_void_p),
                ("mirrors", ctypes.c_void_p), ("n_mirrors", ctypes.c_int)]


class AcefaError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}" if what else STATUS_NAMES.get(status, str(status)))


class Tensor(ctypes.Structure):
    """struct acefa_tensor"""

    _fields_ = [
        ("type", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("nb", ctypes.c_size_t * 4),
        ("data", ctypes.c_void_p),
    ]


_lib = None


def load_library(path: str | None = None):
    """Load libacefa.so (raises OSError if it was not built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise OSError(f"libacefa.so not found at {p}; run acestep.cpp_b200/build.py")
    lib = ctypes.CDLL(p)
    T = ctypes.POINTER(Tensor)
    lib.acefa_flash_attn_ext.argtypes = [T, T, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    lib.acefa_flash_attn_ext.restype = ctypes.c_int
    lib.acefa_workspace_bytes.argtypes = [T, T, T, T, T]
    lib.acefa_workspace_bytes.restype = ctypes.c_size_t
    lib.acefa_supports.argtypes = [T, T, T, T, T, T]
    lib.acefa_supports.restype = ctypes.c_int
    lib.acefa_check.argtypes = [T, T, T, T, T, T]
    lib.acefa_check.restype = ctypes.c_int
    lib.acefa_device_error.argtypes = [ctypes.c_void_p]
    lib.acefa_device_error.restype = ctypes.c_int
    lib.acefa_status_string.argtypes = [ctypes.c_int]
    lib.acefa_status_string.restype = ctypes.c_char_p
    lib.acefa_last_launch_count.restype = ctypes.c_int
    lib.acefa_last_path.restype = ctypes.c_int
    lib.acefa_version.restype = ctypes.c_int
    lib.acefa_flash_attn_ext_noalloc.argtypes = [T, T, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                 ctypes.c_int, ctypes.c_void_p]
    lib.acefa_flash_attn_ext_noalloc.restype = ctypes.c_int
    lib.acefa_flash_attn_ext_mirrored.argtypes = [T, T, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                  ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    lib.acefa_flash_attn_ext_mirrored.restype = ctypes.c_int
    lib.acefa_flash_attn_ext_append.argtypes = [T, T, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                ctypes.c_int, T, T, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_size_t]
    lib.acefa_flash_attn_ext_append.restype = ctypes.c_int
    lib.acefa_flash_attn_ext_gen.argtypes = [T, T, T, ctypes.POINTER(MaskGen), T, T, ctypes.c_float,
                                             ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_size_t]
    lib.acefa_flash_attn_ext_gen.restype = ctypes.c_int
    lib.acefa_flash_attn_ext_fused.argtypes = [T, T, T, T, T, T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                               ctypes.c_int, ctypes.POINTER(OpExt), ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_size_t]
    lib.acefa_flash_attn_ext_fused.restype = ctypes.c_int
    lib.acefa_kv_prologue.argtypes = [T, T, T, T, ctypes.POINTER(RopeNormC), ctypes.c_void_p]
    lib.acefa_kv_prologue.restype = ctypes.c_int
    lib.acefa_cfg_logit_combine.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                            ctypes.c_void_p, ctypes.c_void_p]
    lib.acefa_cfg_logit_combine.restype = ctypes.c_int
    lib.acefa_peer_export.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
    lib.acefa_peer_export.restype = ctypes.c_int
    lib.acefa_peer_import.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
    lib.acefa_peer_import.restype = ctypes.c_int
    lib.acefa_peer_release.argtypes = [ctypes.c_void_p]
    lib.acefa_peer_release.restype = ctypes.c_int
    if path is None:
        _lib = lib
    return lib


def _ggml_type(t: torch.Tensor, gtype: int | None) -> int:
    if gtype is not None:
        return gtype
    if t.dtype == torch.float32:
        return GGML_F32
    if t.dtype == torch.float16:
        return GGML_F16
    if t.dtype == torch.bfloat16:
        return GGML_BF16
    raise TypeError(f"no ggml type for {t.dtype}; pass gtype=GGML_Q8_0 for uint8 Q8_0 blocks")


def describe(t: torch.Tensor | None, gtype: int | None = None, ne0: int | None = None):
    """acefa_tensor for a torch tensor (dims reversed into ggml ne order)."""
    if t is None:
        return None
    if t.dim() > 4:
        raise ValueError("at most 4 dims")
    shape = list(t.shape)[::-1] + [1] * (4 - t.dim())
    es = t.element_size()
    strides = [s * es for s in list(t.stride())[::-1]]
    while len(strides) < 4:
        strides.append(strides[-1] * shape[len(strides) - 1] if strides else es)
    g = _ggml_type(t, gtype)
    d = Tensor()
    d.type = g
    if g == GGML_Q8_0:
        if t.dtype != torch.uint8 or t.stride(-1) != 1:
            raise ValueError("Q8_0 tensors are contiguous uint8 block rows")
        if t.shape[-1] % 34:
            raise ValueError("Q8_0 row bytes must be a multiple of 34")
        shape[0] = ne0 if ne0 is not None else t.shape[-1] // 34 * 32
        strides[0] = 34
    d.ne[:] = shape
    d.nb[:] = strides
    d.data = t.data_ptr()
    return d


def _ref(x):
    return ctypes.byref(x) if x is not None else None


def _stream_ptr(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def result_shape(q: torch.Tensor, v: torch.Tensor, v_type: int | None = None):
    B, Hq, n_q, _ = q.shape
    Dv = v.shape[-1] // 34 * 32 if v_type == GGML_Q8_0 else v.shape[-1]
    return (B, n_q, Hq, Dv)


class Op:
    """One ggml_flash_attn_ext node's operands, described once, callable many times."""

    def __init__(self, q, k, v, mask=None, sinks=None, out=None, kv_type=None, scale=None,
                 max_bias=0.0, softcap=0.0, prec=PREC_F32, mirrors=(), k_new=None, v_new=None, pos=None,
                 mask_gen=None, q_prologue=None, k_prologue=None):
        self.lib = load_library()
        self.q, self.k, self.v, self.mask, self.sinks = q, k, v, mask, sinks
        D = q.shape[-1]
        self.kv_type = kv_type
        if out is None:
            out = torch.empty(result_shape(q, v, kv_type), dtype=torch.float32, device=q.device)
        self.out = out
        self.tq = describe(q)
        self.tk = describe(k, kv_type, D)
        self.tv = describe(v, kv_type, D)
        self.tm = describe(mask, GGML_F16) if mask is not None else None
        self.ts = describe(sinks.reshape(-1), GGML_F32) if sinks is not None else None
        self.td = describe(out)
        self.scale = float(scale if scale is not None else D ** -0.5)
        self.max_bias, self.softcap, self.prec = float(max_bias), float(softcap), int(prec)
        st = self.lib.acefa_check(_ref(self.tq), _ref(self.tk), _ref(self.tv), _ref(self.tm), _ref(self.ts),
                                  _ref(self.td))
        if st != OK:
            raise AcefaError(st, "acefa_check")
        self.ws_bytes = int(self.lib.acefa_workspace_bytes(_ref(self.tq), _ref(self.tk), _ref(self.tv),
                                                           _ref(self.tm), _ref(self.td)))
        self.workspace = torch.empty(max(self.ws_bytes, 256), dtype=torch.uint8, device=q.device)
        # fused KV append: k_new / v_new (Bk, Hkv, 1, D) f32, pos (Bk,) int64 on the device
        self.append = k_new is not None
        if self.append:
            if v_new is None or pos is None or pos.dtype != torch.int64 or not pos.is_cuda:
                raise ValueError("append needs k_new, v_new and an int64 device tensor pos")
            self.k_new, self.v_new, self.pos = k_new, v_new, pos
            self.tkn, self.tvn = describe(k_new), describe(v_new)
        # mask by rule (MaskGen) instead of a mask tensor
        self.mask_gen = mask_gen
        if mask_gen is not None and mask is not None:
            raise ValueError("mask_gen replaces mask")
        # mirrors: device addresses laid out like `out` (e.g. peer GPUs' buffers)
        self.n_mirrors = len(mirrors)
        self.mirrors = (ctypes.c_void_p * max(1, self.n_mirrors))(*[int(m) for m in mirrors])
        # RMSNorm + RoPE prologues (RopeNorm): Q rows, the appended K row
        self.q_prologue, self.k_prologue = q_prologue, k_prologue
        used = [mask_gen is not None, self.append, self.n_mirrors > 0, q_prologue is not None,
                k_prologue is not None]
        self.fused = q_prologue is not None or k_prologue is not None or sum(used) > 1
        if self.fused:
            self.ext = OpExt()
            if mask_gen is not None:
                self.ext.mask_gen = ctypes.addressof(mask_gen)
            if q_prologue is not None:
                self.ext.q_prologue = ctypes.addressof(q_prologue.c)
            if k_prologue is not None:
                self.ext.k_prologue = ctypes.addressof(k_prologue.c)
            if self.append:
                self.ext.k_new, self.ext.v_new = ctypes.addressof(self.tkn), ctypes.addressof(self.tvn)
                self.ext.append_pos = self.pos.data_ptr()
            if self.n_mirrors:
                self.ext.mirrors, self.ext.n_mirrors = ctypes.addressof(self.mirrors), self.n_mirrors

    def __call__(self, stream=None):
        if self.fused:
            st = self.lib.acefa_flash_attn_ext_fused(
                _ref(self.tq), _ref(self.tk), _ref(self.tv), _ref(self.tm), _ref(self.ts), _ref(self.td),
                self.scale, self.max_bias, self.softcap, self.prec, ctypes.byref(self.ext),
                ctypes.c_void_p(_stream_ptr(stream)), ctypes.c_void_p(self.workspace.data_ptr()),
                ctypes.c_size_t(self.workspace.numel()))
            if st != OK:
                raise AcefaError(st, "acefa_flash_attn_ext_fused")
            return self.out
        if self.mask_gen is not None:
            st = self.lib.acefa_flash_attn_ext_gen(
                _ref(self.tq), _ref(self.tk), _ref(self.tv), ctypes.byref(self.mask_gen), _ref(self.ts),
                _ref(self.td), self.scale, self.max_bias, self.softcap, self.prec,
                ctypes.c_void_p(_stream_ptr(stream)), ctypes.c_void_p(self.workspace.data_ptr()),
                ctypes.c_size_t(self.workspace.numel()))
            if st != OK:
                raise AcefaError(st, "acefa_flash_attn_ext_gen")
            return self.out
        if self.append:
            st = self.lib.acefa_flash_attn_ext_append(
                _ref(self.tq), _ref(self.tk), _ref(self.tv), _ref(self.tm), _ref(self.ts), _ref(self.td),
                self.scale, self.max_bias, self.softcap, self.prec, _ref(self.tkn), _ref(self.tvn),
                ctypes.c_void_p(self.pos.data_ptr()), ctypes.c_void_p(_stream_ptr(stream)),
                ctypes.c_void_p(self.workspace.data_ptr()), ctypes.c_size_t(self.workspace.numel()))
            if st != OK:
                raise AcefaError(st, "acefa_flash_attn_ext_append")
            return self.out
        if self.n_mirrors:
            st = self.lib.acefa_flash_attn_ext_mirrored(
                _ref(self.tq), _ref(self.tk), _ref(self.tv), _ref(self.tm), _ref(self.ts), _ref(self.td),
                self.scale, self.max_bias, self.softcap, self.prec, self.mirrors, self.n_mirrors,
                ctypes.c_void_p(_stream_ptr(stream)), ctypes.c_void_p(self.workspace.data_ptr()),
                ctypes.c_size_t(self.workspace.numel()))
            if st != OK:
                raise AcefaError(st, "acefa_flash_attn_ext_mirrored")
            return self.out
        st = self.lib.acefa_flash_attn_ext(
            _ref(self.tq), _ref(self.tk), _ref(self.tv), _ref(self.tm), _ref(self.ts), _ref(self.td),
            self.scale, self.max_bias, self.softcap, self.prec, ctypes.c_void_p(_stream_ptr(stream)),
            ctypes.c_void_p(self.workspace.data_ptr()), ctypes.c_size_t(self.workspace.numel()))
        if st != OK:
            raise AcefaError(st, "acefa_flash_attn_ext")
        return self.out


def flash_attn_ext(q, k, v, mask=None, scale=None, max_bias=0.0, softcap=0.0, sinks=None, kv_type=None,
                   out=None, prec=PREC_F32, stream=None):
    """ggml_flash_attn_ext on the GPU.  Returns dst with torch shape (B, n_q, Hq, Dv)."""
    return Op(q, k, v, mask=mask, sinks=sinks, out=out, kv_type=kv_type, scale=scale, max_bias=max_bias,
              softcap=softcap, prec=prec)(stream)


def supports(q, k, v, mask=None, sinks=None, kv_type=None) -> bool:
    lib = load_library()
    D = q.shape[-1]
    out = torch.empty(0)
    td = Tensor()
    td.type = GGML_F32
    B, Hq, n_q, _ = q.shape
    td.ne[:] = [D, Hq, n_q, B]
    td.nb[:] = [4, 4 * D, 4 * D * Hq, 4 * D * Hq * n_q]
    td.data = 256
    del out
    return bool(lib.acefa_supports(_ref(describe(q)), _ref(describe(k, kv_type, D)), _ref(describe(v, kv_type, D)),
                                   _ref(describe(mask, GGML_F16) if mask is not None else None),
                                   _ref(describe(sinks.reshape(-1), GGML_F32) if sinks is not None else None),
                                   ctypes.byref(td)))


def peer_export(t: torch.Tensor) -> tuple[bytes, int]:
    """CUDA IPC handle of the allocation holding t, and t's byte offset in it."""
    lib = load_library()
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    off = ctypes.c_uint64(0)
    st = lib.acefa_peer_export(ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off))
    if st != OK:
        raise AcefaError(st, "acefa_peer_export")
    return h.raw, int(off.value)


def peer_import(handle: bytes, offset: int) -> int:
    """Map another process's exported buffer; returns its address here."""
    lib = load_library()
    p = ctypes.c_void_p(0)
    st = lib.acefa_peer_import(ctypes.create_string_buffer(handle, PEER_HANDLE_BYTES), ctypes.c_uint64(offset),
                               ctypes.byref(p))
    if st != OK:
        raise AcefaError(st, "acefa_peer_import")
    return int(p.value)


def peer_release(addr: int) -> None:
    st = load_library().acefa_peer_release(ctypes.c_void_p(addr))
    if st != OK:
        raise AcefaError(st, "acefa_peer_release")


def device_error(stream=None) -> int:
    return load_library().acefa_device_error(ctypes.c_void_p(_stream_ptr(stream)))


def last_launch_count() -> int:
    return load_library().acefa_last_launch_count()


def last_path() -> int:
    return load_library().acefa_last_path()


# --------------------------------------------------------------------------
def kv_prologue(k_src, k_dst, v_src=None, v_dst=None, prologue: RopeNorm | None = None, stream=None):
    """acefa_kv_prologue: k_dst = RoPE(RMSNorm(k_src)), v_dst = v_src, converted
    to k_dst's type (f16 / bf16).  Torch shapes (B, H, rows, D), any strides."""
    lib = load_library()
    st = lib.acefa_kv_prologue(_ref(describe(k_src)), _ref(describe(v_src)), _ref(describe(k_dst)),
                               _ref(describe(v_dst)), ctypes.byref(prologue.c) if prologue is not None else None,
                               ctypes.c_void_p(_stream_ptr(stream)))
    if st != OK:
        raise AcefaError(st, "acefa_kv_prologue")
    return k_dst, v_dst


def cfg_logit_combine(cond: torch.Tensor, uncond: torch.Tensor | None, eos_idx: int, code_offset: int,
                      code_count: int, cfg_scale: float, out: torch.Tensor | None = None, stream=None):
    """acefa_cfg_logit_combine: CFG mix + compaction of n logit rows
    (src/pipeline-lm.cpp:471-492).  cond / uncond: (n, row_stride) f32 on the
    device, rows contiguous (uncond None: no CFG).  Returns (n, code_count +
    (eos_idx >= 0)) f32: [EOS, codes...] of uncond + cfg_scale * (cond - uncond)."""
    assert cond.dtype == torch.float32 and cond.dim() == 2 and cond.stride(1) == 1
    n, stride = cond.shape
    if uncond is not None:
        assert uncond.dtype == torch.float32 and uncond.shape == cond.shape and uncond.stride() == cond.stride()
    cols = code_count + (1 if eos_idx >= 0 else 0)
    if out is None:
        out = torch.empty((n, cols), dtype=torch.float32, device=cond.device)
    assert out.is_contiguous() and out.shape == (n, cols)
    lib = load_library()
    st = lib.acefa_cfg_logit_combine(ctypes.c_void_p(cond.data_ptr()),
                                     ctypes.c_void_p(uncond.data_ptr() if uncond is not None else 0),
                                     cond.stride(0), n, eos_idx, code_offset, code_count, cfg_scale,
                                     ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(_stream_ptr(stream)))
    if st != OK:
        raise AcefaError(st, "acefa_cfg_logit_combine")
    return out


# input preparation helpers (torch ops; not on the attention path)

def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    """ggml Q8_0 blocks of x (..., n) -> uint8 (..., n/32*34), bit-exact with
    ggml-quants.c quantize_row_q8_0_ref (d = amax/127 in f32, q = roundf(x/d),
    d stored as f16).  Works on any device; used to build K/V caches."""
    assert x.shape[-1] % 32 == 0
    xb = x.float().reshape(*x.shape[:-1], x.shape[-1] // 32, 32)
    d = xb.abs().amax(dim=-1, keepdim=True) / 127.0
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    y = xb * inv
    a = y.abs()
    fl = torch.floor(a)
    r = torch.sign(y) * (fl + torch.floor(2.0 * (a - fl)))  # round half away from zero
    qs = r.to(torch.int8).view(torch.uint8)
    dh = d.to(torch.float16).view(torch.uint8)  # (..., nb, 2)
    blocks = torch.cat([dh, qs], dim=-1)  # (..., nb, 34)
    return blocks.reshape(*x.shape[:-1], x.shape[-1] // 32 * 34).contiguous()


def dequantize_q8_0(y: torch.Tensor) -> torch.Tensor:
    nb = y.shape[-1] // 34
    b = y.reshape(*y.shape[:-1], nb, 34)
    d = b[..., :2].contiguous().view(torch.float16).float()
    q = b[..., 2:].contiguous().view(torch.int8).float()
    return (q * d).reshape(*y.shape[:-1], nb * 32)
