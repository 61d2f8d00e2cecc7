"""ctypes binding of the CPU oracle (oracle/xn_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline. The product library never imports this module.

Arrays are numpy arrays in their storage type: float32 for f32, uint16 bit
patterns for bf16 and f16. Every function returns a new array.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libxn_oracle.so"

DTYPES = {"f16": 0, "bf16": 1, "f32": 2}
STORAGE = {"f16": np.uint16, "bf16": np.uint16, "f32": np.float32}

_lib = None

_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p


def build(force: bool = False) -> Path:
    """Builds libxn_oracle.so with the committed Makefile (gcc, OpenMP)."""
    src = ORACLE_DIR / "xn_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(ORACLE_DIR), "-B" if force else "all"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "xo_set_num_threads": ([ctypes.c_int], None),
            "xo_get_num_threads": ([], ctypes.c_int),
            "xo_rms_norm": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float], None),
            "xo_layer_norm": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float,
                               ctypes.c_int], None),
            "xo_softmax": ([ctypes.c_int, _c_vp, _c_vp, _c_i64, _c_i64], None),
            "xo_matmul": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int], None),
            "xo_apply_causality_mask": ([ctypes.c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64], None),
            "xo_rope": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64,
                         _c_i64], None),
            "xo_rope_i": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64,
                           _c_i64], None),
            "xo_unary": ([ctypes.c_int, _c_vp, _c_vp, _c_i64, ctypes.c_int], None),
            "xo_binary": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_i64, ctypes.c_int], None),
            "xo_broadcast_binary_rows": ([ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64,
                                          ctypes.c_int], None),
            "xo_index_select": ([_c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64], None),
            "xo_rope_tables": ([ctypes.c_int, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float,
                                ctypes.c_int], None),
            "xo_f32_to_bf16": ([ctypes.c_float], ctypes.c_uint16),
            "xo_bf16_to_f32": ([ctypes.c_uint16], ctypes.c_float),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def set_num_threads(n: int) -> None:
    lib().xo_set_num_threads(int(n))


def get_num_threads() -> int:
    return int(lib().xo_get_num_threads())


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _chk(a: np.ndarray, dtype: str) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype != STORAGE[dtype]:
        raise TypeError(f"oracle: expected storage {STORAGE[dtype]} for {dtype}, got {a.dtype}")
    return a


BINARY_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3}
UNARY_OPS = {"silu": 0, "gelu_erf": 1, "exp": 2}  # "exp": the softmax exp step, cpu_backend.rs:681


def rms_norm(x, alpha, eps: float, dtype: str):
    """cpu_backend.rs:691-709 over the last dimension."""
    x, alpha = _chk(x, dtype), _chk(alpha, dtype)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().xo_rms_norm(DTYPES[dtype], _ptr(out), _ptr(x), _ptr(alpha), cols, x.size // cols, eps)
    return out


def layer_norm(x, w, b, eps: float, dtype: str, remove_mean: bool = True):
    """cpu_backend.rs:711-750 over the last dimension."""
    x, w, b = _chk(x, dtype), _chk(w, dtype), _chk(b, dtype)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().xo_layer_norm(DTYPES[dtype], _ptr(out), _ptr(x), _ptr(w), _ptr(b), cols, x.size // cols, eps,
                        int(remove_mean))
    return out


def softmax(x, dtype: str):
    """cpu_backend.rs:667-689 over the last dimension."""
    x = _chk(x, dtype)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().xo_softmax(DTYPES[dtype], _ptr(out), _ptr(x), cols, x.size // cols)
    return out


def apply_causality_mask(x, offset: int, dtype: str):
    """ops.rs:196-200 (copy, then cpu_backend.rs:647-665 in place) on 3D/4D x."""
    x = _chk(x, dtype).copy()
    if x.ndim == 3:
        bh, t1, t2 = x.shape
    elif x.ndim == 4:
        bh, t1, t2 = x.shape[0] * x.shape[1], x.shape[2], x.shape[3]
    else:
        raise ValueError("apply_causality_mask expects a 3D or 4D tensor")
    lib().xo_apply_causality_mask(DTYPES[dtype], _ptr(x), bh, t1, t2, offset)
    return x


def rope(x, cos, sin, pos: int, dtype: str, interleaved: bool = False):
    """cpu_backend.rs:359-392 (half-split) or :394-422 (interleaved) on [B,H,T,D]."""
    x, cos, sin = _chk(x, dtype), _chk(cos, dtype), _chk(sin, dtype)
    b, h, t, d = x.shape
    out = np.empty_like(x)
    f = lib().xo_rope_i if interleaved else lib().xo_rope
    f(DTYPES[dtype], _ptr(out), _ptr(x), _ptr(cos), _ptr(sin), b, h, t, d, pos)
    return out


def unary(x, op: str, dtype: str):
    """cpu_backend.rs:184-222 for Silu / GeluErf; "exp" is T(exp(x)), the
    per-element step of the softmax (cpu_backend.rs:681)."""
    x = _chk(x, dtype)
    out = np.empty_like(x)
    lib().xo_unary(DTYPES[dtype], _ptr(out), _ptr(x), x.size, UNARY_OPS[op])
    return out


def binary(lhs, rhs, op: str, dtype: str):
    """cpu_backend.rs:224-258."""
    lhs, rhs = _chk(lhs, dtype), _chk(rhs, dtype)
    assert lhs.shape == rhs.shape
    out = np.empty_like(lhs)
    lib().xo_binary(DTYPES[dtype], _ptr(out), _ptr(lhs), _ptr(rhs), lhs.size, BINARY_OPS[op])
    return out


def broadcast_rows(lhs, rhs_row, op: str, dtype: str):
    """cpu_backend.rs:1379-1387: lhs [.., C] op rhs [C] broadcast over rows."""
    lhs, rhs_row = _chk(lhs, dtype), _chk(rhs_row, dtype)
    cols = lhs.shape[-1]
    out = np.empty_like(lhs)
    lib().xo_broadcast_binary_rows(DTYPES[dtype], _ptr(out), _ptr(lhs), _ptr(rhs_row), lhs.size // cols, cols,
                                   BINARY_OPS[op])
    return out


def index_select(x: np.ndarray, ids, dim: int) -> np.ndarray:
    """cpu_backend.rs:624-645 (byte copy) with the output shape of tensor.rs:167-192."""
    x = np.ascontiguousarray(x)
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
    dims = x.shape
    left = int(np.prod(dims[:dim], dtype=np.int64)) if dim > 0 else 1
    right = int(np.prod(dims[dim + 1:], dtype=np.int64)) if dim + 1 < len(dims) else 1
    out_shape = list(dims)
    out_shape[dim] = ids.size
    out = np.empty(out_shape, dtype=x.dtype)
    lib().xo_index_select(x.itemsize, _ptr(out), _ptr(x), _ptr(ids), ids.size, left, dims[dim], right)
    return out


def rope_tables(head_dim: int, max_pos: int, theta: float, dtype: str, variant: str = "mimi"):
    """mimi.rs:1162-1185 (variant "mimi") or llama.rs:406-434 (variant "llama")."""
    half = head_dim // 2
    cos = np.empty((max_pos, half), dtype=STORAGE[dtype])
    sin = np.empty((max_pos, half), dtype=STORAGE[dtype])
    lib().xo_rope_tables(DTYPES[dtype], _ptr(cos), _ptr(sin), head_dim, max_pos, theta,
                         0 if variant == "mimi" else 1)
    return cos, sin


# ---------------------------------------------------------------------------
# Composites: the reference's own op sequences for the fused kernels.
# ---------------------------------------------------------------------------

def residual_prologue(x, branch, layer_scale, dtype: str):
    """h = x + LayerScale(branch): mimi.rs:1199-1201 (broadcast_mul) then
    mimi.rs:1436 (`xs.add(&attn_out)`); without a layer scale, llama.rs:310."""
    if branch is None:
        return x
    t = branch if layer_scale is None else broadcast_rows(branch, layer_scale, "mul", dtype)
    return binary(x, t, "add", dtype)


def rms_norm_residual(x, branch, alpha, eps, dtype, layer_scale=None):
    h = residual_prologue(x, branch, layer_scale, dtype)
    return rms_norm(h, alpha, eps, dtype), h


def layer_norm_residual(x, branch, w, b, eps, dtype, layer_scale=None, remove_mean=True):
    h = residual_prologue(x, branch, layer_scale, dtype)
    return layer_norm(h, w, b, eps, dtype, remove_mean), h


def swiglu(gate, up, dtype: str):
    """llama.rs:256-263: silu(gate) then mul(up)."""
    return binary(unary(gate, "silu", dtype), up, "mul", dtype)


def softmax_causal(x, offset: int, dtype: str):
    """The reference composite: apply_causality_mask then softmax (llama.rs:201-202)."""
    return softmax(apply_causality_mask(x, offset, dtype), dtype)


def rvq_decode(codebooks, codes: np.ndarray, dtype: str, out_layout: str = "bct"):
    """ResidualVectorQuantization::decode (mimi.rs:1730-1744) over codes [B, Q, T]
    as ResidualVectorQuantizer::decode passes them (mimi.rs:1796-1798):
    per codebook, EuclideanCodebook::decode (mimi.rs:1627-1643: ids cast to u32,
    index_select), `.t().contiguous()` (mimi.rs:1689), then `add` in codebook order."""
    b, q, t = codes.shape
    quantized = None
    for i in range(q):
        ids = codes[:, i, :].reshape(-1).astype(np.uint32)
        rows = index_select(codebooks[i], ids, 0).reshape(b, t, -1)
        layer = np.ascontiguousarray(np.swapaxes(rows, 1, 2))  # [B, dim, T]
        quantized = layer if quantized is None else binary(quantized, layer, "add", dtype)
    if out_layout == "btd":
        return np.ascontiguousarray(np.swapaxes(quantized, 1, 2))
    return quantized


# ---------------------------------------------------------------------------
# Streaming decode: the reference's KV cache and attention op sequence.
# ---------------------------------------------------------------------------
def matmul(lhs, rhs, dtype: str, trans_rhs: bool = False):
    """Batched matmul (cpu_backend.rs:45-88 / the gemm crate): lhs [.., m, k]
    times rhs [.., k, n] (or rhs [.., n, k] transposed when trans_rhs, i.e.
    matmul_t); f32 accumulation (sequential in k, FMA), T result."""
    lhs, rhs = _chk(lhs, dtype), _chk(rhs, dtype)
    m, k = lhs.shape[-2:]
    n = rhs.shape[-2] if trans_rhs else rhs.shape[-1]
    assert (rhs.shape[-1] if trans_rhs else rhs.shape[-2]) == k
    batch = int(np.prod(lhs.shape[:-2], dtype=np.int64)) if lhs.ndim > 2 else 1
    assert rhs.shape[:-2] == lhs.shape[:-2]
    out = np.empty(lhs.shape[:-2] + (m, n), dtype=lhs.dtype)
    lib().xo_matmul(DTYPES[dtype], _ptr(out), _ptr(lhs), _ptr(rhs), batch, m, n, k, int(trans_rhs))
    return out


def scale(x, s: float, dtype: str):
    """Tensor::scale (ops.rs:101-105 -> cpu_backend.rs:260-272): T(x * T(s))."""
    x = _chk(x, dtype)
    sv = np.full(x.shape, 0, dtype=x.dtype)
    sv[...] = to_storage_scalar(s, dtype)
    return binary(x, sv, "mul", dtype)


def to_storage_scalar(v: float, dtype: str):
    if dtype == "f32":
        return np.float32(v)
    if dtype == "bf16":
        return np.uint16(lib().xo_f32_to_bf16(float(np.float32(v))))
    return np.float16(np.float32(v)).view(np.uint16)


class KvCacheRef:
    """KvCache::append (mimi-rs/src/models/mimi.rs:1122-1153,
    pocket_tts/src/mimi_transformer.rs:32-61): cat along the sequence axis,
    then keep the last max_seq_len positions. Arrays are [b, h, seq, d]."""

    def __init__(self, max_seq_len: int):
        self.k = self.v = None
        self.max_seq_len = max_seq_len

    def current_seq_len(self) -> int:
        """KvCache::current_seq_len (mimi-rs/src/models/mimi.rs:1115-1120)."""
        return 0 if self.k is None else self.k.shape[2]

    def append(self, k, v):
        if self.k is None:
            nk, nv = k, v
        else:
            nk, nv = np.concatenate([self.k, k], axis=2), np.concatenate([self.v, v], axis=2)
        if nk.shape[2] > self.max_seq_len:
            trim = nk.shape[2] - self.max_seq_len
            nk, nv = nk[:, :, trim:], nv[:, :, trim:]
        self.k, self.v = np.ascontiguousarray(nk), np.ascontiguousarray(nv)
        return self.k, self.v


def split_qkv(qkv, heads: int):
    """The narrow / reshape / transpose / contiguous split of the packed
    in_proj output [b, t, 3*h*d] into q, k, v [b, h, t, d]
    (mimi-rs/src/models/mimi.rs:1330-1346)."""
    b, t, three_hd = qkv.shape
    d = three_hd // (3 * heads)
    parts = qkv.reshape(b, t, 3, heads, d)
    return [np.ascontiguousarray(np.transpose(parts[:, :, i], (0, 2, 1, 3))) for i in range(3)]


def attention_step(q, k, v, scale_value: float, mask_offset: int, dtype: str):
    """The reference attention op sequence on q [b, h, t, d] and the cached
    k, v [b, h, kv, d] (mimi-rs/src/models/mimi.rs:1356-1371): matmul_t,
    scale, apply_causality_mask(mask_offset) (the additive 0 / -inf mask of
    pocket_tts/src/transformer.rs:35-52,138-139 gives the same values with
    mask_offset = kv - t), softmax, matmul; returned as [b, t, h, d]."""
    scores = scale(matmul(q, k, dtype, trans_rhs=True), scale_value, dtype)
    probs = softmax(apply_causality_mask(scores, mask_offset, dtype), dtype)
    out = matmul(probs, v, dtype)
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))
