"""CPU restatement of the Mimi decoder chain (test infrastructure).

TEST INFRASTRUCTURE ONLY: used by tests/ and by bench.py's CPU-baseline leg.

The reference's own op sequence (mimi-rs/src/models/mimi.rs:1317-1445,
1476-1483, 1730-1868), unfused, on the oracle's restatement of the CPU backend
ops. GEMMs are f32 matrix products of the T-typed operands, rounded to T, as
the reference's GEMM returns T values (their summation order is the one thing
no two GEMM libraries share, so the chain is compared with a tolerance).
"""
from __future__ import annotations

import numpy as np

import xn_oracle as oracle_mod


def storage_to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """T storage (f32, or uint16 bits of bf16 / f16) widened to f32."""
    a = np.ascontiguousarray(a)
    if dtype == "f32":
        return a.astype(np.float32)
    if dtype == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


def to_storage(a: np.ndarray, dtype: str) -> np.ndarray:
    """f32 values rounded to T (round-to-nearest-even), as storage."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "f32":
        return a
    if dtype == "f16":
        return a.astype(np.float16).view(np.uint16)
    u = a.view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


class _Widened:
    """Weights widened to f32 once, as a CPU GEMM library keeps them packed."""

    def __init__(self, dtype: str):
        self.dtype, self.cache = dtype, {}

    def __call__(self, b_t: np.ndarray) -> np.ndarray:
        key = id(b_t)
        if key not in self.cache:
            self.cache[key] = (b_t, np.ascontiguousarray(storage_to_f32(b_t, self.dtype).T))
        return self.cache[key][1]


def _mm(a: np.ndarray, b_t: np.ndarray, dtype: str, widened: _Widened | None = None) -> np.ndarray:
    """a [..., K] @ b_t[N, K]^T in f32, rounded to T."""
    bf_t = widened(b_t) if widened is not None else storage_to_f32(b_t, dtype).T
    return to_storage(np.matmul(storage_to_f32(a, dtype), bf_t), dtype)


def _bmm(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    return to_storage(np.matmul(storage_to_f32(a, dtype), storage_to_f32(b, dtype)), dtype)


def rvq_ref(oracle, cfg, w: dict, codes: np.ndarray, dtype: str) -> np.ndarray:
    """SplitResidualVectorQuantizer::decode (mimi-rs/src/models/mimi.rs:1858-1868):
    rvq_first on codebook 0 and rvq_rest on the others, each a gather-sum
    (:1627-1744) and a 1x1 projection (:1796-1806), added in T. codes
    [B, n_q, T] -> [B, T, D]."""
    books = [w[f"quantizer.codebook.{i}"] for i in range(cfg.n_q)]
    first = oracle.rvq_decode(books[:1], np.ascontiguousarray(codes[:, :1]), dtype, "btd")
    x = _mm(first, w["quantizer.rvq_first.output_proj"], dtype)
    if cfg.n_q > 1:
        rest = oracle.rvq_decode(books[1:], np.ascontiguousarray(codes[:, 1:]), dtype, "btd")
        x = oracle.binary(x, _mm(rest, w["quantizer.rvq_rest.output_proj"], dtype), "add", dtype)
    return x


def chain_ref(oracle, cfg, w: dict, cos: np.ndarray, sin: np.ndarray, codes: np.ndarray, dtype: str,
              scale: float) -> np.ndarray:
    # `oracle` is the xn_oracle module (passed explicitly so callers control its build).
    """codes [B, n_q, T] -> [B, T, D]. `w` holds numpy storage arrays keyed as
    mimi_chain.synthetic_weights; `scale` is the T-typed 1/sqrt(head_dim)."""
    B, _, T = codes.shape
    D, H = cfg.d_model, cfg.num_heads
    hd = D // H
    x = rvq_ref(oracle, cfg, w, codes, dtype)
    scale_row = to_storage(np.full(T, scale, dtype=np.float32), dtype)
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        y = oracle.layer_norm(x, w[p + "norm1.weight"], w[p + "norm1.bias"], cfg.eps, dtype)
        qkv = _mm(y, w[p + "self_attn.in_proj_weight"], dtype)
        heads = []
        for part in range(3):
            t = qkv[..., part * D:(part + 1) * D].reshape(B, T, H, hd)
            heads.append(np.ascontiguousarray(np.swapaxes(t, 1, 2)))  # [B, H, T, hd]
        q = oracle.rope(heads[0], cos, sin, 0, dtype, interleaved=True)
        k = oracle.rope(heads[1], cos, sin, 0, dtype, interleaved=True)
        v = heads[2]
        scores = _bmm(q, np.ascontiguousarray(np.swapaxes(k, 2, 3)), dtype)
        scores = oracle.broadcast_rows(scores, scale_row, "mul", dtype)
        probs = oracle.softmax_causal(scores, 0, dtype)
        ctx = _bmm(probs, v, dtype)
        attn = _mm(np.ascontiguousarray(np.swapaxes(ctx, 1, 2)).reshape(B, T, D), w[p + "self_attn.out_proj.weight"],
                   dtype)
        x = oracle.residual_prologue(x, attn, w[p + "layer_scale_1.scale"], dtype)
        y2 = oracle.layer_norm(x, w[p + "norm2.weight"], w[p + "norm2.bias"], cfg.eps, dtype)
        h = _mm(y2, w[p + "linear1.weight"], dtype)
        h = oracle.unary(h, "gelu_erf", dtype)
        m = _mm(h, w[p + "linear2.weight"], dtype)
        x = oracle.residual_prologue(x, m, w[p + "layer_scale_2.scale"], dtype)
    return x


def stream_ref(oracle, cfg, w: dict, cos: np.ndarray, sin: np.ndarray, xs: list, dtype: str, scale: float,
               context: int, act: str = "gelu_erf", mask: str = "absolute", codes: bool = False) -> list:
    """The streaming decoder transformer over a stream of step inputs
    xs[s] = [B, t_s, D]: per layer a cat-then-trim KV cache of `context`
    positions, rope_i, the attention op sequence, LayerNorm / LayerScale /
    residual adds and the MLP (`act` = gelu_erf as Mimi and Pocket, or silu).
    Returns the per-step outputs.

    mask selects the position bookkeeping:
      * "absolute": Pocket's MimiStreamingMultiheadAttention
        (pocket_tts/src/mimi_transformer.rs:114-145): RoPE and
        apply_causality_mask at the absolute position (absolute_offset);
      * "relative": the same with the additive causal mask
        (pocket_tts/src/transformer.rs:35-52), key j visible to query i iff
        j <= i + kv_len - t;
      * "cache_len": mimi-rs's StreamingTransformer::forward
        (mimi-rs/src/models/mimi.rs:1476-1487, 1317-1371): offset = the layer-0
        cache's length before the step (min(total, context)), the RoPE position
        and apply_causality_mask offset of every layer.
    codes=True: each xs[s] is a [B, n_q, t_s] code tensor, decoded by rvq_ref
    first (Mimi::decode_step, mimi.rs:2059-2071, without the conv upsample)."""
    L, D, H = cfg.num_layers, cfg.d_model, cfg.num_heads
    caches = [oracle.KvCacheRef(context) for _ in range(L)]
    total, outs = 0, []
    wide = _Widened(dtype)
    for x in xs:
        if codes:
            x = rvq_ref(oracle, cfg, w, x, dtype)
        B, T, _ = x.shape
        pos = caches[0].current_seq_len() if mask == "cache_len" else total
        for l in range(L):
            p = f"layers.{l}."
            y = oracle.layer_norm(x, w[p + "norm1.weight"], w[p + "norm1.bias"], cfg.eps, dtype)
            q, k, v = oracle.split_qkv(_mm(y, w[p + "self_attn.in_proj_weight"], dtype, wide), H)
            q = oracle.rope(q, cos, sin, pos, dtype, interleaved=True)
            k = oracle.rope(k, cos, sin, pos, dtype, interleaved=True)
            kk, vv = caches[l].append(k, v)
            offset = kk.shape[2] - T if mask == "relative" else pos
            a = oracle.attention_step(q, kk, vv, scale, offset, dtype).reshape(B, T, D)
            attn = _mm(a, w[p + "self_attn.out_proj.weight"], dtype, wide)
            x = oracle.residual_prologue(x, attn, w[p + "layer_scale_1.scale"], dtype)
            y2 = oracle.layer_norm(x, w[p + "norm2.weight"], w[p + "norm2.bias"], cfg.eps, dtype)
            h = oracle.unary(_mm(y2, w[p + "linear1.weight"], dtype, wide), act, dtype)
            x = oracle.residual_prologue(x, _mm(h, w[p + "linear2.weight"], dtype, wide),
                                         w[p + "layer_scale_2.scale"], dtype)
        outs.append(x)
        total += T
    return outs
