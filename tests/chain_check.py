"""Teacher-forced parity of the model chains (tests only).

A chain run with `trace` set records every op's output, GEMM outputs
included. These helpers feed each fused op's exact inputs, as the GPU chain
computed them, to the oracle's restatement of the reference op sequence
(mimi-rs/src/models/mimi.rs:1317-1445; pocket_tts/src/mimi_transformer.rs:
114-145, 232-266) and compare that op's output at the fused-op tolerance
(helpers.assert_close: f32 1e-5 relative, 16-bit 1 ulp, plus the derived
LayerNorm / GELU / attention allowances), and the residual streams, RoPE and
the RVQ gathers bit for bit. GEMMs are the one thing not checked here: they
run on cuBLAS, whose summation order no CPU restatement reproduces.
"""
from __future__ import annotations

import numpy as np

from helpers import (assert_close, attention_abs_bound, from_device, gelu_erf_abs_bound, layer_norm_abs_bound,
                     storage_to_f32)


def collect(trace, dtype: str) -> dict:
    """{(name, layer): numpy storage} of a chain trace (int64 codes as they are)."""
    out = {}
    for name, layer, t in trace:
        out[(name, layer)] = from_device(t, dtype) if t.dtype.is_floating_point else t.cpu().numpy()
    return out


def _ln_allow(h, w, dtype):
    return layer_norm_abs_bound(storage_to_f32(h, dtype), storage_to_f32(w, dtype), 1e-5)


def check_block_tail(oracle, cfg, w, tr: dict, l: int, resid_in, dtype: str, act: str, what: str):
    """The ops of layer l after the attention output projection: LayerScale +
    residual + norm2 (fused), the activation, and LayerScale + residual + the
    next layer's norm1 (fused) or the final LayerScale + residual add.
    Returns the layer's residual output (the next layer's resid_in)."""
    p = f"layers.{l}."
    y2_ref, h_ref = oracle.layer_norm_residual(resid_in, tr[("attn", l)], w[p + "norm2.weight"], w[p + "norm2.bias"],
                                               cfg.eps, dtype, layer_scale=w[p + "layer_scale_1.scale"])
    assert np.array_equal(tr[("resid_mid", l)], h_ref), f"{what} layer {l}: residual after attention differs"
    assert_close(tr[("y2", l)], y2_ref, dtype, f"chain_layer_norm {dtype} {what} layer {l} norm2",
                 extra_abs=_ln_allow(h_ref, w[p + "norm2.weight"], dtype))
    h_pre = tr[("h_pre", l)]
    extra = gelu_erf_abs_bound(storage_to_f32(h_pre, dtype)) if act == "gelu_erf" else None
    assert_close(tr[("h", l)], oracle.unary(h_pre, act, dtype), dtype, f"chain_{act} {dtype} {what} layer {l}",
                 extra_abs=extra)
    m = tr[("m", l)]
    if l + 1 < cfg.num_layers:
        q = f"layers.{l + 1}."
        y_ref, r_ref = oracle.layer_norm_residual(tr[("resid_mid", l)], m, w[q + "norm1.weight"], w[q + "norm1.bias"],
                                                  cfg.eps, dtype, layer_scale=w[p + "layer_scale_2.scale"])
        assert_close(tr[("y", l + 1)], y_ref, dtype, f"chain_layer_norm {dtype} {what} layer {l + 1} norm1",
                     extra_abs=_ln_allow(r_ref, w[q + "norm1.weight"], dtype))
    else:
        r_ref = oracle.residual_prologue(tr[("resid_mid", l)], m, w[p + "layer_scale_2.scale"], dtype)
    assert np.array_equal(tr[("resid", l)], r_ref), f"{what} layer {l}: residual after the MLP differs"
    return r_ref


def check_first_norm(oracle, cfg, w, tr: dict, dtype: str, what: str):
    x = tr[("x", 0)]
    ref = oracle.layer_norm(x, w["layers.0.norm1.weight"], w["layers.0.norm1.bias"], cfg.eps, dtype)
    assert_close(tr[("y", 0)], ref, dtype, f"chain_layer_norm {dtype} {what} layer 0 norm1",
                 extra_abs=_ln_allow(x, w["layers.0.norm1.weight"], dtype))
    return x


def check_rvq(oracle, cfg, w, tr: dict, codes: np.ndarray, dtype: str):
    """The two RVQ gather-sums, bit for bit."""
    books = [w[f"quantizer.codebook.{i}"] for i in range(cfg.n_q)]
    ref = oracle.rvq_decode(books[:1], np.ascontiguousarray(codes[:, :1]), dtype, "btd")
    assert np.array_equal(tr[("rvq_first", -1)], ref), "rvq_first differs"
    if cfg.n_q > 1:
        ref = oracle.rvq_decode(books[1:], np.ascontiguousarray(codes[:, 1:]), dtype, "btd")
        assert np.array_equal(tr[("rvq_rest", -1)], ref), "rvq_rest differs"


def check_whole_sequence(oracle, cfg, w, cos, sin, tr: dict, codes: np.ndarray, dtype: str, scale: float):
    """MimiDecoderChain.decode (offset 0), teacher-forced: the RVQ gather-sums,
    then per layer norm1, the QKV split + rope_i (bit-exact), the scaled
    causal softmax, and the tail of the block."""
    check_rvq(oracle, cfg, w, tr, codes, dtype)
    H = cfg.num_heads
    resid = check_first_norm(oracle, cfg, w, tr, dtype, "whole")
    for l in range(cfg.num_layers):
        q, k, v = oracle.split_qkv(tr[("qkv", l)], H)
        assert np.array_equal(tr[("q", l)], oracle.rope(q, cos, sin, 0, dtype, interleaved=True)), f"layer {l}: q"
        assert np.array_equal(tr[("k", l)], oracle.rope(k, cos, sin, 0, dtype, interleaved=True)), f"layer {l}: k"
        assert np.array_equal(tr[("v", l)], v), f"layer {l}: v"
        scores = tr[("scores", l)]
        scale_row = np.full(scores.shape[-1], oracle.to_storage_scalar(scale, dtype), dtype=scores.dtype)
        ref = oracle.softmax_causal(oracle.broadcast_rows(scores, scale_row, "mul", dtype), 0, dtype)
        assert_close(tr[("probs", l)], ref, dtype, f"chain_softmax {dtype} whole layer {l}")
        resid = check_block_tail(oracle, cfg, w, tr, l, resid, dtype, "gelu_erf", "whole")


def check_stream_step(oracle, cfg, w, cos, sin, tr: dict, caches, total: int, dtype: str, scale: float, act: str,
                      mask: str, what: str):
    """One step of a streaming chain, teacher-forced: norm1 of layer 0, then
    per layer the attention step (split + rope_i at the step's position into
    the reference's cat-then-trim caches, then the attention op sequence, fed
    the GPU's own QKV projection) and the tail of the block. `caches` are the
    oracle KvCacheRef of each layer, carried across steps."""
    H, D = cfg.num_heads, cfg.d_model
    resid = check_first_norm(oracle, cfg, w, tr, dtype, what)
    pos = caches[0].current_seq_len() if mask == "cache_len" else total
    for l in range(cfg.num_layers):
        qkv = tr[("qkv", l)]
        B, T, _ = qkv.shape
        q, k, v = oracle.split_qkv(qkv, H)
        q = oracle.rope(q, cos, sin, pos, dtype, interleaved=True)
        k = oracle.rope(k, cos, sin, pos, dtype, interleaved=True)
        kk, vv = caches[l].append(k, v)
        offset = kk.shape[2] - T if mask == "relative" else pos
        ref = oracle.attention_step(q, kk, vv, scale, offset, dtype).reshape(B, T, D)
        scores = oracle.scale(oracle.matmul(q, kk, dtype, trans_rhs=True), scale, dtype)
        probs = oracle.softmax(oracle.apply_causality_mask(scores, offset, dtype), dtype)
        allow = attention_abs_bound(storage_to_f32(probs, dtype), storage_to_f32(vv, dtype)).reshape(B, T, D)
        assert_close(tr[("a", l)], ref, dtype, f"chain_attention {dtype} {what} layer {l}", extra_abs=allow)
        resid = check_block_tail(oracle, cfg, w, tr, l, resid, dtype, act, what)
