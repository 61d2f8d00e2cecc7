"""Host-side binding of libxn_fused.so, mirroring the `xn` tensor-op API.

The reference exposes these ops as methods of `Tensor<T, B>` in
mimi-rs/src/ops.rs (out-of-place: allocate, then call the in-place form) and
mimi-rs/src/inplace_ops.rs (in-place `*_`: check shapes, then call the
Backend). This module keeps those names, argument meanings and checks, on
torch CUDA tensors, and calls the C ABI declared in include/xn_fused.h. The
fused forms the reference composes from several ops (residual + layer-scale +
norm, SwiGLU, mask + softmax, RVQ decode) are added under new names.

There is no CPU path: every op runs the sm_100a kernels of libxn_fused.so and
raises XnError if the library is missing or a tensor is not on a CUDA device.
torch is used only for device memory and the current stream.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Sequence

import torch

LIB_PATH = Path(__file__).resolve().with_name("libxn_fused.so")

XN_OK, XN_E_INVALID, XN_E_DTYPE, XN_E_RANGE, XN_E_CUDA = 0, 1, 2, 3, 4
XN_UNARY_SILU, XN_UNARY_GELU_ERF = 0, 1
XN_LAYOUT_BHTD, XN_LAYOUT_BTHD = 0, 1
XN_RVQ_MAX_CODEBOOKS = 32
XN_MASK_RELATIVE, XN_MASK_ABSOLUTE, XN_MASK_CACHE_LEN = 0, 1, 2
XN_DEVERR_RANGE, XN_DEVERR_WAIT = 1, 2
MASK_MODES = {"relative": XN_MASK_RELATIVE, "absolute": XN_MASK_ABSOLUTE, "cache_len": XN_MASK_CACHE_LEN}

# Same codes as `enum DType` (mimi-rs/src/dtype.rs:4-10).
DTYPE_CODES = {
    torch.float16: 0,
    torch.bfloat16: 1,
    torch.float32: 2,
    torch.int64: 3,
    torch.uint8: 4,
}
FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


class XnError(RuntimeError):
    """Raised for a failed check or a non-zero status from the C ABI."""

    def __init__(self, msg: str, code: int = XN_E_INVALID):
        super().__init__(msg)
        self.code = code


_lib = None
_vp, _i64, _int, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# Exported C ABI: name -> argtypes (all return int unless listed in _RESTYPE).
SIGNATURES = {
    "xn_last_error": [],
    "xn_abi_version": [],
    "xn_rms_norm": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _int, _vp],
    "xn_layer_norm": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _int, _int, _vp],
    "xn_rope": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _vp],
    "xn_rope_qk": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int,
                   _int, _vp],
    "xn_rope_qk_strided": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                           _int, _int, _vp],
    "xn_unary": [_vp, _vp, _i64, _int, _int, _vp],
    "xn_residual_add": [_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp],
    "xn_softmax_scaled": [_vp, _vp, _i64, _i64, _f32, _int, _i64, _i64, _int, _vp],
    "xn_swiglu": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp],
    "xn_softmax": [_vp, _vp, _i64, _i64, _int, _i64, _i64, _int, _vp],
    "xn_softmax_status": [_vp, _vp, _i64, _i64, _int, _f32, _int, _i64, _i64, _vp, _int, _vp],
    "xn_causality_mask": [_vp, _i64, _i64, _i64, _i64, _int, _vp],
    "xn_index_select": [_vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _int, _vp, _vp],
    "xn_rvq_decode_sum": [_vp, ctypes.POINTER(_vp), _i64, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp,
                          _vp],
    "xn_shard_rows": [_i64, _int, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "xn_kv_append_rope": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _int,
                          _int, _vp, _vp],
    "xn_attention_decode": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _int, _f32,
                            _int, _vp],
    "xn_position_advance": [_vp, _i64, _vp],
    "xn_decode_attention_step": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64,
                                 _i64, _int, _f32, _int, _int, _vp, _vp],
}
_RESTYPE = {"xn_last_error": ctypes.c_char_p}


def lib() -> ctypes.CDLL:
    """Loads libxn_fused.so (fails loudly when it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise XnError(f"{LIB_PATH} is not built: run `python random-things_b200/build.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().xn_last_error().decode()


def _call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != XN_OK:
        raise XnError(f"{name} failed ({rc}): {last_error()}", rc)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dev(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise XnError("xn_fused ops take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise XnError(f"tensors on different devices: {dev} and {t.device}")
        if not t.is_contiguous():
            raise XnError("xn_fused ops take contiguous tensors")
    return dev


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _check_same_shape(a: torch.Size, b: torch.Size, op: str) -> None:
    # inplace_ops.rs check_same_shape
    if tuple(a) != tuple(b):
        raise XnError(f"shape mismatch in {op}, {tuple(a)} <> {tuple(b)}")


def _dtype_code(t: torch.Tensor, floats_only: bool = True) -> int:
    if floats_only and t.dtype not in FLOAT_DTYPES:
        raise XnError(f"unsupported dtype {t.dtype}", XN_E_DTYPE)
    if t.dtype not in DTYPE_CODES:
        raise XnError(f"unsupported dtype {t.dtype}", XN_E_DTYPE)
    return DTYPE_CODES[t.dtype]


def _same_dtype(ref: torch.Tensor, *ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and t.dtype != ref.dtype:
            raise XnError(f"dtype mismatch: {ref.dtype} and {t.dtype}", XN_E_DTYPE)


def _rows_cols(x: torch.Tensor) -> tuple[int, int]:
    # dim_m1 = last dim, d = elem_count / dim_m1 (inplace_ops.rs:264-265)
    cols = x.shape[-1] if x.dim() > 0 else 1
    rows = x.numel() // cols if cols > 0 else 0
    return rows, cols


# ---------------------------------------------------------------------------
# RMSNorm / LayerNorm (inplace_ops.rs:259-307, ops.rs:202-225)
# ---------------------------------------------------------------------------

def rms_norm_(dst: torch.Tensor, src: torch.Tensor, alpha: torch.Tensor, eps: float, *,
              branch: torch.Tensor | None = None, layer_scale: torch.Tensor | None = None,
              residual_out: torch.Tensor | None = None) -> None:
    """In-place RMSNorm (inplace_ops.rs:259-273), optionally fused with
    `h = src + layer_scale * branch` written to residual_out."""
    _check_same_shape(dst.shape, src.shape, "rms_norm_ src")
    if eps <= 0.0:
        raise XnError("rms_norm_ eps must be positive")
    rows, cols = _rows_cols(dst)
    _check_same_shape(alpha.shape, (cols,), "rms_norm_ alpha")
    for name, t in (("branch", branch), ("residual_out", residual_out)):
        if t is not None:
            _check_same_shape(t.shape, src.shape, f"rms_norm_ {name}")
    if layer_scale is not None:
        _check_same_shape(layer_scale.shape, (cols,), "rms_norm_ layer_scale")
    _dev(dst, src, alpha, branch, layer_scale, residual_out)
    _same_dtype(dst, src, alpha, branch, layer_scale, residual_out)
    _call("xn_rms_norm", _p(dst), _p(src), _p(alpha), _p(branch), _p(layer_scale), _p(residual_out),
          rows, cols, float(eps), _dtype_code(dst), _stream(dst))


def rms_norm(x: torch.Tensor, alpha: torch.Tensor, eps: float) -> torch.Tensor:
    """ops.rs:202-207."""
    out = torch.empty_like(x)
    rms_norm_(out, x, alpha, eps)
    return out


def rms_norm_residual(x: torch.Tensor, branch: torch.Tensor, alpha: torch.Tensor, eps: float,
                      layer_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused `h = x + [layer_scale *] branch; y = rms_norm(h)`; returns (y, h)."""
    y, h = torch.empty_like(x), torch.empty_like(x)
    rms_norm_(y, x, alpha, eps, branch=branch, layer_scale=layer_scale, residual_out=h)
    return y, h


def layer_norm_(dst: torch.Tensor, src: torch.Tensor, weight: torch.Tensor | None,
                bias: torch.Tensor | None, eps: float, remove_mean: bool = True, *,
                branch: torch.Tensor | None = None, layer_scale: torch.Tensor | None = None,
                residual_out: torch.Tensor | None = None) -> None:
    """In-place LayerNorm (inplace_ops.rs:275-307) with the optional fused prologue."""
    _check_same_shape(dst.shape, src.shape, "layer_norm_ src")
    if eps <= 0.0:
        raise XnError("layer_norm_ eps must be positive")
    rows, cols = _rows_cols(dst)
    if weight is not None:
        _check_same_shape(weight.shape, (cols,), "layer_norm_ weight")
    if bias is not None:
        _check_same_shape(bias.shape, (cols,), "layer_norm_ bias")
    for name, t in (("branch", branch), ("residual_out", residual_out)):
        if t is not None:
            _check_same_shape(t.shape, src.shape, f"layer_norm_ {name}")
    if layer_scale is not None:
        _check_same_shape(layer_scale.shape, (cols,), "layer_norm_ layer_scale")
    _dev(dst, src, weight, bias, branch, layer_scale, residual_out)
    _same_dtype(dst, src, weight, bias, branch, layer_scale, residual_out)
    _call("xn_layer_norm", _p(dst), _p(src), _p(weight), _p(bias), _p(branch), _p(layer_scale),
          _p(residual_out), rows, cols, float(eps), int(bool(remove_mean)), _dtype_code(dst), _stream(dst))


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """ops.rs:210-212."""
    return layer_norm_rm(x, weight, bias, eps, True)


def layer_norm_rm(x, weight, bias, eps: float, remove_mean: bool) -> torch.Tensor:
    """ops.rs:215-225."""
    out = torch.empty_like(x)
    layer_norm_(out, x, weight, bias, eps, remove_mean)
    return out


def layer_norm_residual(x: torch.Tensor, branch: torch.Tensor, weight, bias, eps: float,
                        layer_scale: torch.Tensor | None = None,
                        remove_mean: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused `h = x + [layer_scale *] branch; y = layer_norm(h)`; returns (y, h).
    Replaces mimi.rs:1433-1439 (LayerScale, add, norm2)."""
    y, h = torch.empty_like(x), torch.empty_like(x)
    layer_norm_(y, x, weight, bias, eps, remove_mean, branch=branch, layer_scale=layer_scale,
                residual_out=h)
    return y, h


# ---------------------------------------------------------------------------
# RoPE (inplace_ops.rs:421-473, ops.rs:227-239)
# ---------------------------------------------------------------------------

def _rope_dims(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: int, layout: str, op: str):
    _check_same_shape(cos.shape, sin.shape, f"{op} cos/sin")
    if x.dim() != 4:
        raise XnError(f"{op}: expected a 4D tensor, got shape {tuple(x.shape)}")
    if cos.dim() != 2:
        raise XnError(f"{op}: expected 2D cos/sin tables, got shape {tuple(cos.shape)}")
    if layout == "bhtd":
        b, h, t, d = x.shape
    elif layout == "bthd":
        b, t, h, d = x.shape
    else:
        raise XnError(f"{op}: unknown layout {layout!r}")
    max_pos, d_over_2 = cos.shape
    if d_over_2 * 2 != d:
        raise XnError(f"{op} requires even d dimension, got d={d}, {tuple(x.shape)} {tuple(cos.shape)}")
    if pos + t > max_pos:
        raise XnError(f"{op} position out of range, pos={pos} + t={t} > max_pos={max_pos}", XN_E_RANGE)
    return b, h, t, d, max_pos


def rope_(dst: torch.Tensor, src: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: int, *,
          interleaved: bool = False, layout: str = "bhtd") -> None:
    """In-place RoPE: rope_ (inplace_ops.rs:421-446) or, with interleaved=True,
    rope_i_ (inplace_ops.rs:448-473). layout="bthd" takes [B, T, H, D] directly."""
    op = "rope_i_" if interleaved else "rope_"
    _check_same_shape(dst.shape, src.shape, f"{op} src")
    b, h, t, d, max_pos = _rope_dims(dst, cos, sin, pos, layout, op)
    _dev(dst, src, cos, sin)
    _same_dtype(dst, src, cos, sin)
    _call("xn_rope", _p(dst), _p(src), _p(cos), _p(sin), b, h, t, d, int(pos), max_pos, int(interleaved),
          XN_LAYOUT_BHTD if layout == "bhtd" else XN_LAYOUT_BTHD, _dtype_code(dst), _stream(dst))


def rope(x, cos, sin, pos: int, layout: str = "bhtd") -> torch.Tensor:
    """ops.rs:228-232 (half-split)."""
    out = torch.empty_like(x)
    rope_(out, x, cos, sin, pos, interleaved=False, layout=layout)
    return out


def rope_i(x, cos, sin, pos: int, layout: str = "bhtd") -> torch.Tensor:
    """ops.rs:235-239 (interleaved)."""
    out = torch.empty_like(x)
    rope_(out, x, cos, sin, pos, interleaved=True, layout=layout)
    return out


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos, sin, pos: int, *, interleaved: bool = False,
            layout: str = "bhtd", out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """Q and K rotated by one launch (mimi.rs:1350-1351, llama.rs:171-172)."""
    op = "rope_qk"
    bq, hq, tq, dq, max_pos = _rope_dims(q, cos, sin, pos, layout, op)
    bk, hk, tk, dk, _ = _rope_dims(k, cos, sin, pos, layout, op)
    if (bq, tq, dq) != (bk, tk, dk):
        raise XnError(f"{op}: q {tuple(q.shape)} and k {tuple(k.shape)} differ outside the head dim")
    qo, ko = out if out is not None else (torch.empty_like(q), torch.empty_like(k))
    _check_same_shape(qo.shape, q.shape, f"{op} q out")
    _check_same_shape(ko.shape, k.shape, f"{op} k out")
    _dev(q, k, cos, sin, qo, ko)
    _same_dtype(q, k, cos, sin, qo, ko)
    _call("xn_rope_qk", _p(qo), _p(q), _p(ko), _p(k), _p(cos), _p(sin), bq, hq, hk, tq, dq, int(pos), max_pos,
          int(interleaved), XN_LAYOUT_BHTD if layout == "bhtd" else XN_LAYOUT_BTHD, _dtype_code(q), _stream(q))
    return qo, ko


def rope_qk_packed(qkv: torch.Tensor, heads: int, cos, sin, pos: int, *, kv_heads: int | None = None,
                   interleaved: bool = True, out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """RoPE on the Q and K parts of a packed [B, T, (H + 2*Hkv) * D] projection
    (mimi.rs:1326-1351: narrow, reshape, transpose, contiguous, then rope_i),
    read in place. Returns rotated (q, k) as contiguous [B, T, H, D] / [B, T, Hkv, D]."""
    op = "rope_qk_packed"
    if qkv.dim() != 3 or not qkv.is_contiguous():
        raise XnError(f"{op}: expected a contiguous [B, T, C] projection, got {tuple(qkv.shape)}")
    kv_heads = heads if kv_heads is None else kv_heads
    b, t, c = qkv.shape
    if c % (heads + 2 * kv_heads):
        raise XnError(f"{op}: width {c} is not (heads + 2 * kv_heads) * d")
    d = c // (heads + 2 * kv_heads)
    _check_same_shape(cos.shape, sin.shape, f"{op} cos/sin")
    max_pos, d_over_2 = cos.shape
    if d_over_2 * 2 != d:
        raise XnError(f"{op} requires even d dimension, got d={d}")
    if pos + t > max_pos:
        raise XnError(f"{op} position out of range, pos={pos} + t={t} > max_pos={max_pos}", XN_E_RANGE)
    qo, ko = out if out is not None else (
        torch.empty((b, t, heads, d), dtype=qkv.dtype, device=qkv.device),
        torch.empty((b, t, kv_heads, d), dtype=qkv.dtype, device=qkv.device))
    if heads != kv_heads:
        raise XnError(f"{op}: outputs share one token stride; use heads == kv_heads")
    _dev(qkv, cos, sin, qo, ko)
    _same_dtype(qkv, cos, sin, qo, ko)
    esz = qkv.element_size()
    k_src = qkv.data_ptr() + heads * d * esz
    _call("xn_rope_qk_strided", _p(qo), _p(qkv), _p(ko), k_src, _p(cos), _p(sin), b, heads, kv_heads, t, d,
          int(pos), max_pos, c, heads * d, int(interleaved), _dtype_code(qkv), _stream(qkv))
    return qo, ko


# ---------------------------------------------------------------------------
# Activations (inplace_ops.rs unary_, ops.rs:178-182,458-464)
# ---------------------------------------------------------------------------

def unary_(dst: torch.Tensor, src: torch.Tensor, op: str) -> None:
    codes = {"silu": XN_UNARY_SILU, "gelu_erf": XN_UNARY_GELU_ERF}
    if op not in codes:
        raise XnError(f"unary_: unsupported op {op!r}")
    _check_same_shape(dst.shape, src.shape, f"{op}_")
    _dev(dst, src)
    _same_dtype(dst, src)
    _call("xn_unary", _p(dst), _p(src), dst.numel(), codes[op], _dtype_code(dst), _stream(dst))


def silu(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    unary_(out, x, "silu")
    return out


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    unary_(out, x, "gelu_erf")
    return out


def residual_add_(dst: torch.Tensor, x: torch.Tensor, branch: torch.Tensor,
                  layer_scale: torch.Tensor | None = None) -> None:
    """dst = x + layer_scale * branch (LayerScale then add, mimi.rs:1441-1444)."""
    _check_same_shape(x.shape, branch.shape, "residual_add_ branch")
    _check_same_shape(dst.shape, x.shape, "residual_add_ dst")
    rows, cols = _rows_cols(dst)
    if layer_scale is not None:
        _check_same_shape(layer_scale.shape, (cols,), "residual_add_ layer_scale")
    _dev(dst, x, branch, layer_scale)
    _same_dtype(dst, x, branch, layer_scale)
    _call("xn_residual_add", _p(dst), _p(x), _p(branch), _p(layer_scale), rows, cols, _dtype_code(dst),
          _stream(dst))


def residual_add(x: torch.Tensor, branch: torch.Tensor, layer_scale: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x)
    residual_add_(out, x, branch, layer_scale)
    return out


def swiglu_(dst: torch.Tensor, gate: torch.Tensor, up: torch.Tensor) -> None:
    """dst = silu(gate) * up over the last dimension; gate / up may be
    last-dim slices of one packed projection (row stride >= cols)."""
    if gate.shape != up.shape or dst.shape != gate.shape:
        raise XnError(f"swiglu_: shape mismatch {tuple(dst.shape)} {tuple(gate.shape)} {tuple(up.shape)}")
    _dev(dst)
    for t in (gate, up):
        if not t.is_cuda or t.device != dst.device:
            raise XnError("swiglu_: tensors must be on the same CUDA device")
        if t.dim() == 0 or t.stride(-1) != 1 or not _rows_uniform(t):
            raise XnError("swiglu_: gate/up must have unit last-dim stride and uniformly strided rows")
    _same_dtype(dst, gate, up)
    rows, cols = _rows_cols(dst)
    gs = gate.stride(-2) if gate.dim() > 1 else cols
    us = up.stride(-2) if up.dim() > 1 else cols
    _call("xn_swiglu", _p(dst), _p(gate), _p(up), rows, cols, gs, us, _dtype_code(dst), _stream(dst))


def _rows_uniform(t: torch.Tensor) -> bool:
    # All leading dims collapse into one row dimension of stride t.stride(-2).
    if t.dim() <= 2:
        return True
    expect = t.stride(-2) * t.shape[-2]
    for i in range(t.dim() - 3, -1, -1):
        if t.shape[i] != 1 and t.stride(i) != expect:
            return False
        expect *= t.shape[i]
    return True


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up (llama.rs:256-263) in one pass."""
    out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    swiglu_(out, gate, up)
    return out


# ---------------------------------------------------------------------------
# Softmax and causal mask (inplace_ops.rs:230-257, ops.rs:184-200)
# ---------------------------------------------------------------------------

def _mask_dims(x: torch.Tensor, op: str) -> tuple[int, int, int]:
    if x.dim() == 3:
        return x.shape[0], x.shape[1], x.shape[2]
    if x.dim() == 4:
        return x.shape[0] * x.shape[1], x.shape[2], x.shape[3]
    raise XnError(f"{op} expects 3D or 4D tensor, got shape {tuple(x.shape)}")


def softmax_(dst: torch.Tensor, src: torch.Tensor) -> None:
    """inplace_ops.rs:230-238."""
    _check_same_shape(dst.shape, src.shape, "softmax_")
    _dev(dst, src)
    _same_dtype(dst, src)
    rows, cols = _rows_cols(dst)
    _call("xn_softmax", _p(dst), _p(src), rows, cols, 0, 1, 0, _dtype_code(dst), _stream(dst))


def softmax(x: torch.Tensor) -> torch.Tensor:
    """ops.rs:185-189."""
    out = torch.empty_like(x)
    softmax_(out, x)
    return out


def softmax_causal_(dst: torch.Tensor, src: torch.Tensor, offset: int) -> None:
    """apply_causality_mask(offset) followed by softmax, fused; masked entries
    are not read and come out as exactly 0."""
    _check_same_shape(dst.shape, src.shape, "softmax_causal_")
    bh, t1, t2 = _mask_dims(src, "softmax_causal_")
    _dev(dst, src)
    _same_dtype(dst, src)
    _call("xn_softmax", _p(dst), _p(src), bh * t1, t2, 1, max(t1, 1), int(offset), _dtype_code(dst),
          _stream(dst))


def softmax_causal(x: torch.Tensor, offset: int) -> torch.Tensor:
    out = torch.empty_like(x)
    softmax_causal_(out, x, offset)
    return out


def attn_softmax_(dst: torch.Tensor, scores: torch.Tensor, scale: float, offset: int | None = None) -> None:
    """softmax(mask(T(scores * scale))) over the last dimension: the score
    scale, optional causal mask (offset given) and softmax of mimi.rs:1361-1368
    in one pass. `scale` is the T-typed scale value."""
    _check_same_shape(dst.shape, scores.shape, "attn_softmax_")
    _dev(dst, scores)
    _same_dtype(dst, scores)
    if offset is None:
        rows, cols = _rows_cols(dst)
        _call("xn_softmax_scaled", _p(dst), _p(scores), rows, cols, float(scale), 0, 1, 0, _dtype_code(dst),
              _stream(dst))
    else:
        bh, t1, t2 = _mask_dims(scores, "attn_softmax_")
        _call("xn_softmax_scaled", _p(dst), _p(scores), bh * t1, t2, float(scale), 1, max(t1, 1), int(offset),
              _dtype_code(dst), _stream(dst))


def attn_softmax(scores: torch.Tensor, scale: float, offset: int | None = None) -> torch.Tensor:
    out = torch.empty_like(scores)
    attn_softmax_(out, scores, scale, offset)
    return out


def softmax_status_(dst: torch.Tensor, src: torch.Tensor, err_flag: torch.Tensor, *, scale: float | None = None,
                    offset: int | None = None) -> None:
    """softmax_ / attn_softmax_ (scale and causal offset optional) that also
    reports, in the int32 device word err_flag, XN_DEVERR_WAIT when a bounded
    wait of the wide-row kernel gave up (its unfinished rows are then NaN)."""
    _check_same_shape(dst.shape, src.shape, "softmax_status_")
    _dev(dst, src, err_flag)
    _same_dtype(dst, src)
    if err_flag.dtype != torch.int32:
        raise XnError("softmax_status_: err_flag must be an int32 CUDA tensor")
    if offset is None:
        rows, cols = _rows_cols(dst)
        causal, t1, off = 0, 1, 0
    else:
        bh, t1, cols = _mask_dims(src, "softmax_status_")
        rows, causal, off = bh * t1, 1, int(offset)
    _call("xn_softmax_status", _p(dst), _p(src), rows, cols, 0 if scale is None else 1,
          1.0 if scale is None else float(scale), causal, max(t1, 1), off, _p(err_flag), _dtype_code(dst),
          _stream(dst))


def apply_causality_mask_(x: torch.Tensor, offset: int) -> None:
    """inplace_ops.rs:244-257."""
    bh, t1, t2 = _mask_dims(x, "apply_causality_mask")
    _dev(x)
    _call("xn_causality_mask", _p(x), bh, t1, t2, int(offset), _dtype_code(x), _stream(x))


def apply_causality_mask(x: torch.Tensor, offset: int) -> torch.Tensor:
    """ops.rs:196-200 (copy, then mask in place)."""
    out = x.clone()
    apply_causality_mask_(out, offset)
    return out


# ---------------------------------------------------------------------------
# Gathers (tensor.rs:166-192, cpu_backend.rs:624-645; mimi.rs:1627-1744)
# ---------------------------------------------------------------------------

def _ids_tensor(ids, device) -> tuple[torch.Tensor, int]:
    if isinstance(ids, torch.Tensor):
        if not ids.is_cuda or ids.device != device:
            raise XnError("index_select: ids must be a CUDA tensor on the source's device")
        if ids.dtype == torch.int64:
            return ids.contiguous(), 1
        if ids.dtype in (torch.int32, torch.uint32):
            return ids.contiguous(), 0
        raise XnError(f"index_select: ids dtype {ids.dtype} (expected int32/uint32/int64)")
    t = torch.as_tensor(list(ids), dtype=torch.int64).to(device)
    return t, 1


def index_select(x: torch.Tensor, ids, dim: int, *, err_flag: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Tensor::index_select (tensor.rs:167-192) with device-resident ids.
    Host-side ids (a Python sequence) are bounds-checked on the host first, as
    the reference does (tensor.rs:170-176); device ids are checked on the device:
    an out-of-range id yields a zero row and sets err_flag[0] = 1."""
    _dev(x)
    if dim < 0:
        dim += x.dim()
    if not 0 <= dim < x.dim():
        raise XnError(f"index_select: dim {dim} out of range for shape {tuple(x.shape)}")
    dim_size = x.shape[dim]
    if not isinstance(ids, torch.Tensor):
        ids = list(ids)
        for i, idx in enumerate(ids):
            if idx < 0 or idx >= dim_size:
                raise XnError(f"index_select: index {idx} at position {i} is out of bounds for dimension "
                              f"{dim} with size {dim_size}")
    ids_t, is_i64 = _ids_tensor(ids, x.device)
    n_ids = ids_t.numel()
    out_shape = list(x.shape)
    out_shape[dim] = n_ids
    if out is None:
        out = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    else:
        _check_same_shape(out.shape, out_shape, "index_select out")
        _dev(out)
        _same_dtype(x, out)
    left = 1
    for s in x.shape[:dim]:
        left *= s
    right = 1
    for s in x.shape[dim + 1:]:
        right *= s
    if err_flag is not None:
        _dev(err_flag)
        if err_flag.dtype != torch.int32:
            raise XnError("index_select: err_flag must be an int32 CUDA tensor")
    _call("xn_index_select", _p(out), _p(x), _p(ids_t), is_i64, n_ids, left, dim_size, right,
          _dtype_code(x, floats_only=False), _p(err_flag), _stream(x))
    return out


def rvq_decode_sum(codebooks: Sequence[torch.Tensor], codes: torch.Tensor, *, out_layout: str = "bct",
                   err_flag: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused RVQ decode over codes [B, Q, T] (int64) and Q codebooks [bins, dim]:
    the sum over codebooks of the selected rows, as [B, dim, T] ("bct", the
    layout of ResidualVectorQuantization::decode, mimi.rs:1730-1744) or
    [B, T, dim] ("btd")."""
    if codes.dim() != 3 or codes.dtype != torch.int64:
        raise XnError("rvq_decode_sum: codes must be an int64 [B, Q, T] tensor")
    b, q, t = codes.shape
    if q != len(codebooks) or not 1 <= q <= XN_RVQ_MAX_CODEBOOKS:
        raise XnError(f"rvq_decode_sum: {len(codebooks)} codebooks for {q} code rows "
                      f"(at most {XN_RVQ_MAX_CODEBOOKS})")
    bins, dim = codebooks[0].shape
    for cb in codebooks:
        if tuple(cb.shape) != (bins, dim):
            raise XnError("rvq_decode_sum: codebooks must share one [bins, dim] shape")
    _dev(codes, *codebooks)
    _same_dtype(codebooks[0], *codebooks)
    shape = (b, dim, t) if out_layout == "bct" else (b, t, dim)
    if out_layout not in ("bct", "btd"):
        raise XnError(f"rvq_decode_sum: unknown layout {out_layout!r}")
    if out is None:
        out = torch.empty(shape, dtype=codebooks[0].dtype, device=codes.device)
    else:
        _check_same_shape(out.shape, shape, "rvq_decode_sum out")
        _dev(out)
        _same_dtype(codebooks[0], out)
    tables = (ctypes.c_void_p * q)(*[cb.data_ptr() for cb in codebooks])
    if err_flag is not None:
        _dev(err_flag)
    _call("xn_rvq_decode_sum", _p(out), tables, q, _p(codes), b, t, dim, bins, int(out_layout == "bct"),
          _dtype_code(out), _p(err_flag), _stream(out))
    return out


# ---------------------------------------------------------------------------
# Streaming decode: ring-buffer KV cache (mimi.rs:1099-1153, 1317-1384;
# pocket_tts/src/transformer.rs, mimi_transformer.rs)
# ---------------------------------------------------------------------------

def _total_args(total: int | None, total_dev: torch.Tensor | None, op: str) -> tuple[int, int | None]:
    if total_dev is not None:
        if total_dev.dtype != torch.int64 or total_dev.numel() != 1 or not total_dev.is_cuda:
            raise XnError(f"{op}: total_dev must be a one-element int64 CUDA tensor")
        return 0, total_dev.data_ptr()
    if total is None or total < 0:
        raise XnError(f"{op}: need total >= 0 or total_dev")
    return int(total), None


def kv_append_rope(qkv: torch.Tensor, heads: int, cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, total: int | None = None, *, interleaved: bool = True,
                   total_dev: torch.Tensor | None = None, err_flag: torch.Tensor | None = None,
                   q_out: torch.Tensor | None = None) -> torch.Tensor:
    """Splits the packed projection qkv [B, T, 3*H*D], applies RoPE (rope_i when
    interleaved, as mimi.rs:1350-1351 and pocket_tts/src/rope.rs) to q and k at
    positions total + i, writes k and v into the ring caches [B, H, cap, D] at
    slots (total + i) % cap, and returns q as [B, H, T, D]. With total_dev
    (int64 [1] on the device) the position is read on the device."""
    op = "kv_append_rope"
    if qkv.dim() != 3 or not qkv.is_contiguous():
        raise XnError(f"{op}: expected a contiguous [B, T, 3*H*D] projection, got {tuple(qkv.shape)}")
    b, t, c = qkv.shape
    if c % (3 * heads):
        raise XnError(f"{op}: width {c} is not 3 * heads * d")
    d = c // (3 * heads)
    if k_cache.dim() != 4 or tuple(k_cache.shape) != (b, heads, k_cache.shape[2], d):
        raise XnError(f"{op}: k_cache must be [B, H, cap, D] = [{b}, {heads}, cap, {d}], got {tuple(k_cache.shape)}")
    _check_same_shape(k_cache.shape, v_cache.shape, f"{op} caches")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise XnError(f"{op}: caches must be contiguous")
    _check_same_shape(cos.shape, sin.shape, f"{op} cos/sin")
    max_pos, d_over_2 = cos.shape
    if d_over_2 * 2 != d:
        raise XnError(f"{op} requires even d dimension, got d={d}")
    tot, tdev = _total_args(total, total_dev, op)
    if tdev is None and tot + t > max_pos:
        raise XnError(f"{op} position out of range, pos={tot} + t={t} > max_pos={max_pos}", XN_E_RANGE)
    if q_out is None:
        q_out = torch.empty((b, heads, t, d), dtype=qkv.dtype, device=qkv.device)
    else:
        _check_same_shape(q_out.shape, (b, heads, t, d), f"{op} q_out")
    _dev(qkv, cos, sin, k_cache, v_cache, q_out)
    _same_dtype(qkv, cos, sin, k_cache, v_cache, q_out)
    if err_flag is not None:
        _dev(err_flag)
        if err_flag.dtype != torch.int32:
            raise XnError(f"{op}: err_flag must be an int32 CUDA tensor")
    _call("xn_kv_append_rope", _p(q_out), _p(k_cache), _p(v_cache), _p(qkv), _p(cos), _p(sin), b, heads, t, d,
          tot, tdev, max_pos, k_cache.shape[2], int(interleaved), _dtype_code(qkv), _p(err_flag), _stream(qkv))
    return q_out


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, total: int | None,
                     context: int, scale: float, *, mask: str = "relative", total_dev: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of q [B, H, T, D] over the last min(total + T, context) cached
    positions: scale, causal mask ("relative": key j <= i + kv_len - T as
    pocket_tts/src/transformer.rs:35-52; "absolute": j <= total + i as
    apply_causality_mask(offset) in mimi.rs:1364), softmax and the weighted sum
    of V, as the reference's op sequence (mimi.rs:1356-1371). Returns
    [B, T, H*D] (the out_proj input)."""
    op = "attention_decode"
    if q.dim() != 4 or not q.is_contiguous():
        raise XnError(f"{op}: q must be a contiguous [B, H, T, D] tensor")
    b, h, t, d = q.shape
    if k_cache.dim() != 4 or tuple(k_cache.shape[:2]) != (b, h) or k_cache.shape[3] != d:
        raise XnError(f"{op}: k_cache must be [B, H, cap, D] = [{b}, {h}, cap, {d}], got {tuple(k_cache.shape)}")
    _check_same_shape(k_cache.shape, v_cache.shape, f"{op} caches")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise XnError(f"{op}: caches must be contiguous")
    if mask not in MASK_MODES:
        raise XnError(f"{op}: unknown mask mode {mask!r}")
    tot, tdev = _total_args(total, total_dev, op)
    if out is None:
        out = torch.empty((b, t, h * d), dtype=q.dtype, device=q.device)
    elif out.numel() != b * t * h * d or not out.is_contiguous():
        raise XnError(f"{op}: out must be a contiguous [B, T, H*D] tensor")
    _dev(q, k_cache, v_cache, out)
    _same_dtype(q, k_cache, v_cache, out)
    _call("xn_attention_decode", _p(out), _p(q), _p(k_cache), _p(v_cache), b, h, t, d, tot, tdev,
          k_cache.shape[2], int(context), MASK_MODES[mask], float(scale), _dtype_code(q), _stream(q))
    return out


def decode_attention_step(qkv: torch.Tensor, heads: int, cos: torch.Tensor, sin: torch.Tensor,
                          k_cache: torch.Tensor, v_cache: torch.Tensor, total: int | None, context: int,
                          scale: float, *, interleaved: bool = True, mask: str = "relative",
                          total_dev: torch.Tensor | None = None, err_flag: torch.Tensor | None = None,
                          out: torch.Tensor | None = None) -> torch.Tensor:
    """kv_append_rope followed by attention_decode in one launch (q stays on
    chip): the step's attention output [B, T, H*D] from the packed projection
    qkv [B, T, 3*H*D], with the caches updated as kv_append_rope does.
    mask "cache_len" is mimi-rs's StreamingTransformer (mimi.rs:1476-1487):
    the new rows rotate at the cache's length before the step,
    min(total, context), which is also the mask offset."""
    op = "decode_attention_step"
    if qkv.dim() != 3 or not qkv.is_contiguous():
        raise XnError(f"{op}: expected a contiguous [B, T, 3*H*D] projection, got {tuple(qkv.shape)}")
    b, t, c = qkv.shape
    if c % (3 * heads):
        raise XnError(f"{op}: width {c} is not 3 * heads * d")
    d = c // (3 * heads)
    if k_cache.dim() != 4 or tuple(k_cache.shape) != (b, heads, k_cache.shape[2], d):
        raise XnError(f"{op}: k_cache must be [B, H, cap, D] = [{b}, {heads}, cap, {d}], got {tuple(k_cache.shape)}")
    _check_same_shape(k_cache.shape, v_cache.shape, f"{op} caches")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise XnError(f"{op}: caches must be contiguous")
    _check_same_shape(cos.shape, sin.shape, f"{op} cos/sin")
    max_pos, d_over_2 = cos.shape
    if d_over_2 * 2 != d:
        raise XnError(f"{op} requires even d dimension, got d={d}")
    if mask not in MASK_MODES:
        raise XnError(f"{op}: unknown mask mode {mask!r}")
    tot, tdev = _total_args(total, total_dev, op)
    # The new rows rotate at total + i, or at min(total, context) + i ("cache_len").
    rope0 = min(tot, int(context)) if mask == "cache_len" else tot
    if tdev is None and rope0 + t > max_pos:
        raise XnError(f"{op} position out of range, pos={rope0} + t={t} > max_pos={max_pos}", XN_E_RANGE)
    if out is None:
        out = torch.empty((b, t, heads * d), dtype=qkv.dtype, device=qkv.device)
    elif out.numel() != b * t * heads * d or not out.is_contiguous():
        raise XnError(f"{op}: out must be a contiguous [B, T, H*D] tensor")
    _dev(qkv, cos, sin, k_cache, v_cache, out)
    _same_dtype(qkv, cos, sin, k_cache, v_cache, out)
    if err_flag is not None:
        _dev(err_flag)
        if err_flag.dtype != torch.int32:
            raise XnError(f"{op}: err_flag must be an int32 CUDA tensor")
    _call("xn_decode_attention_step", _p(out), _p(k_cache), _p(v_cache), _p(qkv), _p(cos), _p(sin), b, heads, t,
          d, tot, tdev, max_pos, k_cache.shape[2], int(context), MASK_MODES[mask], float(scale), int(interleaved),
          _dtype_code(qkv), _p(err_flag), _stream(qkv))
    return out


def position_advance(total_dev: torch.Tensor, t: int) -> None:
    """total_dev += t on the device (the end of a captured decode step)."""
    _total_args(None, total_dev, "position_advance")
    _call("xn_position_advance", _p(total_dev), int(t), _stream(total_dev))


# ---------------------------------------------------------------------------
# Row sharding across GPUs (no reference counterpart; the reference is 1-GPU)
# ---------------------------------------------------------------------------

def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """(first_row, count) of this rank's contiguous block of ceil(rows/world) rows."""
    b, c = ctypes.c_int64(), ctypes.c_int64()
    _call("xn_shard_rows", int(rows), int(world), int(rank), ctypes.byref(b), ctypes.byref(c))
    return b.value, c.value


def all_gather_rows(local: torch.Tensor, rows: int, group=None) -> torch.Tensor:
    """Optional all-gather of row shards into the full [rows, ...] tensor on
    every rank (NCCL over NVLink on GPUs, gloo on CPU). Only called when a
    caller asks for the full output; the sharded ops need no collective."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    per = -(-rows // world) if world > 0 else 0
    tail = local.shape[1:]
    if local.shape[0] == per and local.is_contiguous():
        padded = local  # an even split needs no padding copy
    else:
        padded = torch.zeros((per, *tail), dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        full = torch.empty((per * world, *tail), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, padded, group=group)
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
        full = torch.cat(parts, dim=0)
    return full[:rows]
