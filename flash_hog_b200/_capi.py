"""ctypes binding of the C ABI in ``include/flash_hog_b200.h``.

This is the counterpart of the reference's plugin loader
(``flash_hog/jax/_tk_gpu.py:30-58``): it loads the in-tree shared library with
ctypes (``FLASH_HOG_B200_LIB`` overrides the path, as ``FLASH_HOG_TK_LIB``
does there) and exposes one thin wrapper per entry point taking torch CUDA
tensors. There is no fallback: if the library is missing or a call fails, an
exception is raised.
"""

from __future__ import annotations

import ctypes
import functools
import os

import torch

_LIB_ENV = "FLASH_HOG_B200_LIB"
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libflashhog_b200.so")

FH_OK = 0
STATUS_NAMES = {
    0: "FH_OK",
    1: "FH_ERR_INVALID_ARGUMENT",
    2: "FH_ERR_UNSUPPORTED",
    3: "FH_ERR_LAUNCH",
    4: "FH_ERR_DEVICE",
    5: "FH_ERR_INJECTED",
    6: "FH_ERR_NO_DEVICE",
}

# Every symbol include/flash_hog_b200.h declares.
EXPORTED_SYMBOLS = (
    "fh_attn_fwd",
    "fh_attn_rowdot",
    "fh_attn_bwd",
    "fh_attn_bwdbwd",
    "fh_attn_bwdbwd_pass",
    "fh_attn_bwdbwd_o",
    "fh_attn_bwdbwd_noalloc",
    "fh_attn_jvp_bwd",
    "fh_attn_fwd_f32",
    "fh_attn_bwd_f32",
    "fh_attn_bwdbwd_f32",
    "fh_attn_jvp_bwd_f32",
    "fh_layernorm_scratch_floats",
    "fh_layernorm_fwd",
    "fh_layernorm_bwd",
    "fh_layernorm_bwd_bwd",
    "fh_gelu",
    "fh_xent_fwd",
    "fh_xent_bwd",
    "fh_xent_bwd_bwd",
    "fh_device_status",
    "fh_status_string",
    "fh_last_error",
    "fh_abi_version",
    "fh_launch_count",
)
ABI_VERSION = 8


class FlashHogError(RuntimeError):
    """A C ABI call returned a non-zero status."""

    def __init__(self, entry: str, status: int, message: str):
        super().__init__(f"{entry}: {STATUS_NAMES.get(status, status)} ({message})")
        self.entry = entry
        self.status = status


class FhStrides(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("head", ctypes.c_int64)]


class FhAttnDims(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seq_q", ctypes.c_int32),
        ("seq_k", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("q", FhStrides),
        ("k", FhStrides),
        ("kv_heads", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_k", ctypes.c_void_p),
        ("max_seqlen_q", ctypes.c_int32),
        ("max_seqlen_k", ctypes.c_int32),
    ]


def library_path() -> str:
    return os.environ.get(_LIB_ENV) or _LIB_PATH


@functools.cache
def lib() -> ctypes.CDLL:
    path = library_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"flash_hog_b200 CUDA library not found at {path}; build it with `python -m flash_hog_b200.build`")
    h = ctypes.CDLL(path)
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    dims = ctypes.POINTER(FhAttnDims)
    h.fh_attn_fwd.argtypes = [vp, dims, vp, vp, vp, vp, vp, f32, i32]
    h.fh_attn_rowdot.argtypes = [vp, dims, vp, vp, vp]
    h.fh_attn_bwd.argtypes = [vp, dims, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, f32, i32]
    h.fh_attn_bwdbwd.argtypes = [vp, dims] + [vp] * 15 + [f32, i32]
    h.fh_attn_bwdbwd_pass.argtypes = [vp, dims] + [vp] * 15 + [f32, i32, i32]
    h.fh_attn_bwdbwd_o.argtypes = [vp, dims] + [vp] * 16 + [f32, i32, i32]
    h.fh_attn_bwdbwd_noalloc.argtypes = [vp, dims] + [vp] * 13 + [f32, i32, vp]
    h.fh_attn_jvp_bwd.argtypes = [vp, dims] + [vp] * 17 + [f32, i32]
    h.fh_attn_fwd_f32.argtypes = [vp, dims] + [vp] * 5 + [f32, i32]
    h.fh_attn_bwd_f32.argtypes = [vp, dims] + [vp] * 10 + [f32, i32]
    h.fh_attn_bwdbwd_f32.argtypes = [vp, dims] + [vp] * 16 + [f32, i32, i32]
    h.fh_attn_jvp_bwd_f32.argtypes = [vp, dims] + [vp] * 17 + [f32, i32]
    h.fh_layernorm_scratch_floats.argtypes = [i32, i32]
    h.fh_layernorm_scratch_floats.restype = ctypes.c_longlong
    h.fh_layernorm_fwd.argtypes = [vp, i32, i32, vp, vp, vp, f32, vp, vp, vp]
    h.fh_layernorm_bwd.argtypes = [vp, i32, i32] + [vp] * 9
    h.fh_layernorm_bwd_bwd.argtypes = [vp, i32, i32] + [vp] * 12
    h.fh_gelu.argtypes = [vp, i32, i32, ctypes.c_longlong, vp, vp, vp, vp, vp]
    ll = ctypes.c_longlong
    h.fh_xent_fwd.argtypes = [vp, i32, i32, i32, ll, vp, vp, vp, vp]
    h.fh_xent_bwd.argtypes = [vp, i32, i32, i32, ll, vp, vp, vp, vp, f32, vp]
    h.fh_xent_bwd_bwd.argtypes = [vp, i32, i32, i32, ll, vp, vp, vp, vp, f32, vp, vp, vp]
    h.fh_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
    h.fh_status_string.argtypes = [i32]
    h.fh_status_string.restype = ctypes.c_char_p
    h.fh_abi_version.argtypes = []
    h.fh_launch_count.argtypes = []
    h.fh_launch_count.restype = ctypes.c_ulonglong
    h.fh_last_error.argtypes = []
    h.fh_last_error.restype = ctypes.c_char_p
    for name in ("fh_attn_fwd", "fh_attn_rowdot", "fh_attn_bwd", "fh_attn_bwdbwd", "fh_attn_bwdbwd_pass",
                 "fh_attn_bwdbwd_o", "fh_attn_bwdbwd_noalloc", "fh_attn_jvp_bwd", "fh_attn_fwd_f32",
                 "fh_attn_bwd_f32", "fh_attn_bwdbwd_f32", "fh_attn_jvp_bwd_f32", "fh_device_status",
                 "fh_abi_version", "fh_layernorm_fwd", "fh_layernorm_bwd", "fh_layernorm_bwd_bwd", "fh_gelu",
                 "fh_xent_fwd", "fh_xent_bwd", "fh_xent_bwd_bwd"):
        getattr(h, name).restype = i32
    if h.fh_abi_version() != ABI_VERSION:
        raise RuntimeError(f"flash_hog_b200 ABI mismatch: library {h.fh_abi_version()}, binding {ABI_VERSION}")
    return h


def _check(entry: str, rc: int) -> None:
    if rc != FH_OK:
        detail = lib().fh_last_error().decode()
        msg = lib().fh_status_string(rc).decode() + (f": {detail}" if detail else "")
        raise FlashHogError(entry, rc, msg)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _strides(t: torch.Tensor) -> FhStrides:
    """(batch, seq, head) element strides; a size-1 dimension is never stepped
    over, so its stride is normalised (torch leaves it arbitrary)."""
    (sb, st, sh, sd), (b, tq, h, d) = t.stride(), t.shape
    if sd != 1 and d > 1:
        raise ValueError("head_dim must be the contiguous dimension")
    return FhStrides(sb if b > 1 else 0, st if tq > 1 else 8, sh if h > 1 else 0)


def _layout_key(t: torch.Tensor):
    s = _strides(t)
    return tuple(t.shape), (s.batch, s.seq, s.head)


class Varlen:
    """A packed variable-length batch for the C ABI: int32 device offsets
    ``cu_seqlens_q``/``cu_seqlens_k`` (sequences + 1 entries) and the longest
    sequence lengths. The tensors are then (1, total rows, heads, head_dim)."""

    def __init__(self, cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int,
                 max_seqlen_k: int):
        for name, c in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
            if c.dtype != torch.int32 or c.ndim != 1 or not c.is_contiguous() or c.numel() < 2:
                raise ValueError(f"{name} must be a contiguous 1-D int32 tensor of sequences + 1 offsets")
        if cu_seqlens_q.numel() != cu_seqlens_k.numel():
            raise ValueError("cu_seqlens_q and cu_seqlens_k must describe the same number of sequences")
        self.cu_seqlens_q, self.cu_seqlens_k = cu_seqlens_q, cu_seqlens_k
        self.max_seqlen_q, self.max_seqlen_k = int(max_seqlen_q), int(max_seqlen_k)

    @property
    def batch(self) -> int:
        return self.cu_seqlens_q.numel() - 1


def make_dims(q: torch.Tensor, k: torch.Tensor, window: int = 0, varlen: Varlen | None = None) -> FhAttnDims:
    """Dims for BTNH tensors: q (B, Tq, H, D), k (B, Tk, Hkv, D) with H a multiple of
    Hkv; ``window`` is the sliding-window length of a causal mask (0 = unlimited).
    With ``varlen`` the tensors are packed (1, total, H, D) sequences."""
    b, tq, h, d = q.shape
    tk, hkv = k.shape[1], k.shape[2]
    dims = FhAttnDims(b, h, tq, tk, d, _strides(q), _strides(k), hkv, int(window))
    if varlen is not None:
        if b != 1:
            raise ValueError("packed variable-length tensors have one batch entry: (1, total, heads, head_dim)")
        if varlen.cu_seqlens_q.device != q.device or varlen.cu_seqlens_k.device != q.device:
            raise ValueError("cu_seqlens must be on the tensors' device")
        dims.batch = varlen.batch
        dims.cu_seqlens_q = varlen.cu_seqlens_q.data_ptr()
        dims.cu_seqlens_k = varlen.cu_seqlens_k.data_ptr()
        dims.max_seqlen_q, dims.max_seqlen_k = varlen.max_seqlen_q, varlen.max_seqlen_k
    return dims


def _same_layout(ref: torch.Tensor, *others: torch.Tensor, dtype=torch.bfloat16) -> None:
    """Checks shape, strides, dtype and device against ``ref`` (None entries,
    unused outputs, are skipped)."""
    for t in (ref,) + others:
        if t is None:
            continue
        if _layout_key(t) != _layout_key(ref):
            raise ValueError("tensors of one side must share shape and strides")
        if t.dtype != dtype or t.device != ref.device:
            raise ValueError(f"tensors must be {dtype} on the same CUDA device")


def attn_fwd(q, k, v, out, lse, scale: float, causal: int, window: int = 0, varlen: Varlen | None = None) -> None:
    _same_layout(q, out)
    _same_layout(k, v)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_fwd", lib().fh_attn_fwd(_stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v),
                                           _ptr(out), _ptr(lse), float(scale), int(causal)))


def attn_rowdot(o, dO, delta, varlen: Varlen | None = None) -> None:
    _same_layout(o, dO)
    dims = make_dims(o, o, 0, varlen)
    _check("fh_attn_rowdot", lib().fh_attn_rowdot(_stream(o.device), ctypes.byref(dims), _ptr(o), _ptr(dO),
                                                 _ptr(delta)))


def attn_bwd(q, k, v, o, dO, lse, dq, dk, dv, delta, scale: float, causal: int, window: int = 0, varlen: Varlen | None = None) -> None:
    _same_layout(q, o, dO, dq)
    _same_layout(k, v, dk, dv)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_bwd", lib().fh_attn_bwd(_stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v),
                                           _ptr(o), _ptr(dO), _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv),
                                           _ptr(delta), float(scale), int(causal)))


def attn_bwdbwd(q, k, v, dO, ddq, ddk, ddv, lse, delta, dq2, ddo, dk2, dv2, dd, bvec, scale: float,
                causal: int, window: int = 0, varlen: Varlen | None = None) -> None:
    _same_layout(q, dO, ddq, dq2, ddo)
    _same_layout(k, v, ddk, ddv, dk2, dv2)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_bwdbwd", lib().fh_attn_bwdbwd(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(dO), _ptr(ddq), _ptr(ddk),
        _ptr(ddv), _ptr(lse), _ptr(delta), _ptr(dq2), _ptr(ddo), _ptr(dk2), _ptr(dv2), _ptr(dd), _ptr(bvec),
        float(scale), int(causal)))


PASS_QUERY, PASS_KEY, PASS_FWD_TANGENT = 1, 2, 4


def attn_bwdbwd_pass(q, k, v, dO, ddq, ddk, ddv, lse, delta, dq2, ddo, dk2, dv2, dd, bvec, scale: float,
                     causal: int, which: int, window: int = 0, varlen: Varlen | None = None) -> None:
    """One pass of the double backward (PASS_QUERY, PASS_KEY or both)."""
    _same_layout(q, dO, ddq, dq2, ddo)
    _same_layout(k, v, ddk, ddv, dk2, dv2)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_bwdbwd_pass", lib().fh_attn_bwdbwd_pass(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(dO), _ptr(ddq), _ptr(ddk),
        _ptr(ddv), _ptr(lse), _ptr(delta), _ptr(dq2), _ptr(ddo), _ptr(dk2), _ptr(dv2), _ptr(dd), _ptr(bvec),
        float(scale), int(causal), int(which)))


def attn_bwdbwd_o(q, k, v, o, dO, ddq, ddk, ddv, lse, dq2, ddo, dk2, dv2, delta, dd, bvec, scale: float,
                  causal: int, which: int = PASS_QUERY | PASS_KEY, window: int = 0, varlen: Varlen | None = None) -> None:
    """Double backward from the forward output: the query pass computes delta itself."""
    _same_layout(q, o, dO, ddq, dq2, ddo)
    _same_layout(k, v, ddk, ddv, dk2, dv2)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_bwdbwd_o", lib().fh_attn_bwdbwd_o(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(ddq),
        _ptr(ddk), _ptr(ddv), _ptr(lse), _ptr(dq2), _ptr(ddo), _ptr(dk2), _ptr(dv2), _ptr(delta), _ptr(dd),
        _ptr(bvec), float(scale), int(causal), int(which)))


def attn_jvp_bwd(q, k, v, o, dO, lse, tq, tk, tv, tdO, tdq, tdk, tdv, to, delta, dd, bvec, scale: float,
                 causal: int, window: int = 0, varlen: Varlen | None = None) -> None:
    """Forward-mode derivative of the first-order backward (``tdO`` may be None)."""
    _same_layout(q, o, dO, tq, tdq, to, tdO)
    _same_layout(k, v, tk, tv, tdk, tdv)
    dims = make_dims(q, k, window, varlen)
    _check("fh_attn_jvp_bwd", lib().fh_attn_jvp_bwd(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(lse), _ptr(tq),
        _ptr(tk), _ptr(tv), _ptr(tdO), _ptr(tdq), _ptr(tdk), _ptr(tdv), _ptr(to),
        _ptr(delta), _ptr(dd), _ptr(bvec), float(scale), int(causal)))


_F32 = torch.float32


def attn_fwd_f32(q, k, v, out, lse, scale: float, causal: int, window: int = 0) -> None:
    """``attn_fwd`` with fp32 tensors, fp32 products (``fh_attn_fwd_f32``)."""
    _same_layout(q, out, dtype=_F32)
    _same_layout(k, v, dtype=_F32)
    dims = make_dims(q, k, window)
    _check("fh_attn_fwd_f32", lib().fh_attn_fwd_f32(_stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k),
                                                   _ptr(v), _ptr(out), _ptr(lse), float(scale), int(causal)))


def attn_bwd_f32(q, k, v, o, dO, lse, dq, dk, dv, delta, scale: float, causal: int, window: int = 0) -> None:
    """``attn_bwd`` with fp32 tensors (``fh_attn_bwd_f32``)."""
    _same_layout(q, o, dO, dq, dtype=_F32)
    _same_layout(k, v, dk, dv, dtype=_F32)
    dims = make_dims(q, k, window)
    _check("fh_attn_bwd_f32", lib().fh_attn_bwd_f32(_stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k),
                                                   _ptr(v), _ptr(o), _ptr(dO), _ptr(lse), _ptr(dq), _ptr(dk),
                                                   _ptr(dv), _ptr(delta), float(scale), int(causal)))


def attn_bwdbwd_f32(q, k, v, o, dO, ddq, ddk, ddv, lse, dq2, ddo, dk2, dv2, delta, dd, bvec, scale: float,
                    causal: int, which: int = PASS_QUERY | PASS_KEY, window: int = 0) -> None:
    """``attn_bwdbwd_o`` with fp32 tensors (``fh_attn_bwdbwd_f32``)."""
    _same_layout(q, o, dO, ddq, dq2, ddo, dtype=_F32)
    _same_layout(k, v, ddk, ddv, dk2, dv2, dtype=_F32)
    dims = make_dims(q, k, window)
    _check("fh_attn_bwdbwd_f32", lib().fh_attn_bwdbwd_f32(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(ddq),
        _ptr(ddk), _ptr(ddv), _ptr(lse), _ptr(dq2), _ptr(ddo), _ptr(dk2), _ptr(dv2), _ptr(delta), _ptr(dd),
        _ptr(bvec), float(scale), int(causal), int(which)))


def attn_jvp_bwd_f32(q, k, v, o, dO, lse, tq, tk, tv, tdO, tdq, tdk, tdv, to, delta, dd, bvec, scale: float,
                     causal: int, window: int = 0) -> None:
    """``attn_jvp_bwd`` with fp32 tensors (``fh_attn_jvp_bwd_f32``)."""
    _same_layout(q, o, dO, tq, tdq, to, tdO, dtype=_F32)
    _same_layout(k, v, tk, tv, tdk, tdv, dtype=_F32)
    dims = make_dims(q, k, window)
    _check("fh_attn_jvp_bwd_f32", lib().fh_attn_jvp_bwd_f32(
        _stream(q.device), ctypes.byref(dims), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(lse), _ptr(tq),
        _ptr(tk), _ptr(tv), _ptr(tdO), _ptr(tdq), _ptr(tdk), _ptr(tdv), _ptr(to),
        _ptr(delta), _ptr(dd), _ptr(bvec), float(scale), int(causal)))


def _ln_rows(x: torch.Tensor, cols: int) -> int:
    if x.dtype != torch.float32 or not x.is_contiguous() or x.shape[-1] != cols:
        raise ValueError("layernorm tensors are contiguous fp32 (..., cols)")
    return x.numel() // cols


def layernorm_scratch(rows: int, cols: int, device) -> torch.Tensor:
    with torch.cuda.device(device):
        n = int(lib().fh_layernorm_scratch_floats(int(rows), int(cols)))
    if n < 0:
        _check("fh_layernorm_scratch_floats", 2)
    return torch.empty(n, dtype=torch.float32, device=device)


def layernorm_fwd(x, w, b, eps: float, y, mean, rstd) -> None:
    cols = w.numel()
    rows = _ln_rows(x, cols)
    _check("fh_layernorm_fwd", lib().fh_layernorm_fwd(_stream(x.device), rows, cols, _ptr(x), _ptr(w), _ptr(b),
                                                     float(eps), _ptr(y), _ptr(mean), _ptr(rstd)))


def layernorm_bwd(x, w, mean, rstd, dy, dx, dw, db) -> None:
    cols = w.numel()
    rows = _ln_rows(x, cols)
    scratch = layernorm_scratch(rows, cols, x.device)
    _check("fh_layernorm_bwd", lib().fh_layernorm_bwd(_stream(x.device), rows, cols, _ptr(x), _ptr(w), _ptr(mean),
                                                     _ptr(rstd), _ptr(dy), _ptr(dx), _ptr(dw), _ptr(db),
                                                     _ptr(scratch)))


def layernorm_bwd_bwd(x, w, mean, rstd, dy, ddx, ddw, ddb, gx, gw, gdy) -> None:
    """Cotangents ddx, ddw, ddb may be None (zero)."""
    cols = w.numel()
    rows = _ln_rows(x, cols)
    scratch = layernorm_scratch(rows, cols, x.device)
    _check("fh_layernorm_bwd_bwd", lib().fh_layernorm_bwd_bwd(
        _stream(x.device), rows, cols, _ptr(x), _ptr(w), _ptr(mean), _ptr(rstd), _ptr(dy), _ptr(ddx), _ptr(ddw),
        _ptr(ddb), _ptr(gx), _ptr(gw), _ptr(gdy), _ptr(scratch)))


_GELU_DTYPES = {torch.float32: 0, torch.bfloat16: 1}


def gelu(mode: int, a, dh, c, out0, out1) -> None:
    """Exact GELU (mode 0), its backward (1) or its backward's backward (2); see fh_gelu."""
    if a.dtype not in _GELU_DTYPES or not a.is_contiguous():
        raise ValueError("gelu tensors are contiguous fp32 or bf16")
    for t in (dh, c, out0, out1):
        if t is not None and (t.dtype != a.dtype or not t.is_contiguous() or t.numel() != a.numel()):
            raise ValueError("gelu tensors must share dtype, size and contiguity")
    _check("fh_gelu", lib().fh_gelu(_stream(a.device), int(mode), _GELU_DTYPES[a.dtype], a.numel(), _ptr(a), _ptr(dh),
                                   _ptr(c), _ptr(out0), _ptr(out1)))


def _xent_args(z, t):
    if z.dim() != 2 or z.dtype not in _GELU_DTYPES or z.stride(1) != 1:
        raise ValueError("xent logits are a (rows, vocab) fp32 or bf16 tensor with unit column stride")
    if t.dtype != torch.int64 or not t.is_contiguous() or t.numel() != z.shape[0]:
        raise ValueError("xent targets are a contiguous int64 vector of one entry per row")
    return _GELU_DTYPES[z.dtype], z.shape[0], z.shape[1], z.stride(0)


def xent_fwd(z, t, lse, loss) -> None:
    """Per-row log-sum-exp and loss of (rows, vocab) logits; see fh_xent_fwd."""
    dt, rows, vocab, ld = _xent_args(z, t)
    _check("fh_xent_fwd", lib().fh_xent_fwd(_stream(z.device), dt, rows, vocab, ld, _ptr(z), _ptr(t), _ptr(lse),
                                             _ptr(loss)))


def xent_bwd(z, t, lse, g, s: float, dz) -> None:
    """dz = g s (softmax(z) - onehot(t)); g a one-element fp32 device tensor."""
    dt, rows, vocab, ld = _xent_args(z, t)
    if dz.dtype != z.dtype or not dz.is_contiguous() or dz.shape != z.shape:
        raise ValueError("dz is a contiguous tensor of the logits' shape and dtype")
    _check("fh_xent_bwd", lib().fh_xent_bwd(_stream(z.device), dt, rows, vocab, ld, _ptr(z), _ptr(t), _ptr(lse),
                                             _ptr(g), float(s), _ptr(dz)))


def xent_bwd_bwd(z, t, lse, g, s: float, u, gz, gg) -> None:
    """Backward's backward given the cotangent u of dz; see fh_xent_bwd_bwd."""
    dt, rows, vocab, ld = _xent_args(z, t)
    for x in (u, gz):
        if x.dtype != z.dtype or not x.is_contiguous() or x.shape != z.shape:
            raise ValueError("u and gz are contiguous tensors of the logits' shape and dtype")
    _check("fh_xent_bwd_bwd", lib().fh_xent_bwd_bwd(_stream(z.device), dt, rows, vocab, ld, _ptr(z), _ptr(t),
                                                     _ptr(lse), _ptr(g), float(s), _ptr(u), _ptr(gz), _ptr(gg)))


def launch_count() -> int:
    """Kernels launched by the library in this process so far."""
    return int(lib().fh_launch_count())


def device_status(device=None) -> int:
    """Synchronises the current stream and returns (and clears) the device error code."""
    code = ctypes.c_int(0)
    lib().fh_device_status(_stream(device), ctypes.byref(code))
    return int(code.value)
