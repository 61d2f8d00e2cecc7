"""Mimi decoder chain on the fused ops: RVQ decode + decoder transformer.

This is the caller the fused layer ops were built for. It restates, for the
ops on the path, the reference's
  * SplitResidualVectorQuantizer::decode (mimi-rs/src/models/mimi.rs:1858-1868)
    -> ResidualVectorQuantizer::decode (:1796-1806, 1x1-conv output projection)
    -> ResidualVectorQuantization::decode (:1730-1744) -> codebook gathers,
  * StreamingTransformer::forward (:1476-1483) over StreamingTransformerLayer
    (:1423-1445) with StreamingMultiheadAttention (:1317-1384) and Mlp
    (:1256-1269), norm_first, LayerNorm (eps 1e-5), LayerScale, interleaved
    RoPE, causal softmax, GELU(erf),
with every layer op on the sm_100a kernels and the layer-to-layer glue fused:
  * the two RVQ codebook loops -> two xn_rvq_decode_sum launches,
  * LayerScale + residual add + next LayerNorm -> one xn_layer_norm,
  * narrow/transpose/contiguous + rope_i on Q and K -> one xn_rope_qk_strided
    reading the packed QKV projection,
  * scale + causal mask + softmax -> one xn_softmax_scaled,
  * the final LayerScale + add -> one xn_residual_add.
GEMMs (projections, attention products, MLP) run on cuBLAS through
torch.matmul, as the reference runs them on cuBLAS. The SEANet decoder and the
upsampling transposed convolution are outside this path; the chain runs the
decoder transformer at the codes' frame rate on [B, T, D] (the reference's
conv_layout transposes, :1528-1548, become layout choices).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

import xn_fused as xn


@dataclass
class MimiChainConfig:
    """The Mimi v0.1 values used on this path (mimi.rs:1908-1963)."""

    d_model: int = 512
    num_heads: int = 8
    num_layers: int = 8
    dim_feedforward: int = 2048
    max_period: float = 10000.0
    max_seq_len: int = 8192
    context: int = 250
    n_q: int = 8
    bins: int = 2048
    q_dim: int = 256
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


def rope_tables(cfg: MimiChainConfig, dtype: torch.dtype, device) -> tuple[torch.Tensor, torch.Tensor]:
    """RotaryEmbedding::new (mimi.rs:1162-1185): inv_freq = 1 / theta^(i / half),
    angle = pos * inv_freq, evaluated in f32 and rounded to T."""
    half = cfg.head_dim // 2
    i = torch.arange(half, dtype=torch.float32)
    inv = 1.0 / torch.pow(torch.tensor(cfg.max_period, dtype=torch.float32), i / half)
    ang = torch.arange(cfg.max_seq_len, dtype=torch.float32)[:, None] * inv[None, :]
    return ang.cos().to(dtype).to(device), ang.sin().to(dtype).to(device)


def synthetic_weights(cfg: MimiChainConfig, dtype: torch.dtype, device, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded random weights with the reference's tensor names and shapes.
    Codebook entries ~ N(0, 1), layer scales ~ U(0, 0.1), norm gains ~ N(1, 0.02),
    projections ~ N(0, 1/fan_in) so activations stay O(1)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    D, F, Q = cfg.d_model, cfg.dim_feedforward, cfg.q_dim

    def n(shape, std=1.0, mean=0.0):
        return (torch.randn(shape, generator=g) * std + mean).to(dtype).to(device)

    def u(shape, hi):
        return (torch.rand(shape, generator=g) * hi).to(dtype).to(device)

    w: dict[str, torch.Tensor] = {}
    for i in range(cfg.n_q):
        w[f"quantizer.codebook.{i}"] = n((cfg.bins, Q))
    w["quantizer.rvq_first.output_proj"] = n((D, Q), 1 / math.sqrt(Q))
    w["quantizer.rvq_rest.output_proj"] = n((D, Q), 1 / math.sqrt(Q))
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        w[p + "norm1.weight"] = n(D, 0.02, 1.0)
        w[p + "norm1.bias"] = n(D, 0.02)
        w[p + "self_attn.in_proj_weight"] = n((3 * D, D), 1 / math.sqrt(D))
        w[p + "self_attn.out_proj.weight"] = n((D, D), 1 / math.sqrt(D))
        w[p + "layer_scale_1.scale"] = u(D, 0.1)
        w[p + "norm2.weight"] = n(D, 0.02, 1.0)
        w[p + "norm2.bias"] = n(D, 0.02)
        w[p + "linear1.weight"] = n((F, D), 1 / math.sqrt(D))
        w[p + "linear2.weight"] = n((D, F), 1 / math.sqrt(F))
        w[p + "layer_scale_2.scale"] = u(D, 0.1)
    return w


class MimiDecoderChain:
    """RVQ decode + decoder transformer over whole sequences (offset 0)."""

    def __init__(self, cfg: MimiChainConfig, weights: dict[str, torch.Tensor], cos: torch.Tensor,
                 sin: torch.Tensor):
        self.cfg, self.w, self.cos, self.sin = cfg, weights, cos, sin
        dtype = weights["quantizer.codebook.0"].dtype
        # StreamingMultiheadAttention: T::from_f32(1 / sqrt(head_dim)) (mimi.rs:1361).
        self.scale = float(torch.tensor(1.0 / math.sqrt(cfg.head_dim), dtype=torch.float32).to(dtype).float())
        self.books = [weights[f"quantizer.codebook.{i}"] for i in range(cfg.n_q)]
        # When a list, every op's inputs and outputs are appended to it as
        # (name, layer, tensor copy): the tests check each fused op on the
        # exact inputs it received (GEMM outputs included).
        self.trace: list | None = None

    def _rec(self, name: str, layer: int, t: torch.Tensor) -> None:
        if self.trace is not None:
            self.trace.append((name, layer, t.detach().clone()))

    # -- RVQ ---------------------------------------------------------------
    def rvq_decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n_q, T] (int64) -> embeddings [B, T, D]: rvq_first on
        codebook 0 plus rvq_rest on codebooks 1.., each a gather-sum and a 1x1
        projection, then added in T."""
        w = self.w
        first = xn.rvq_decode_sum(self.books[:1], codes[:, :1].contiguous(), out_layout="btd")
        x = torch.matmul(first, w["quantizer.rvq_first.output_proj"].t())
        self._rec("rvq_first", -1, first)
        if self.cfg.n_q > 1:
            rest = xn.rvq_decode_sum(self.books[1:], codes[:, 1:].contiguous(), out_layout="btd")
            self._rec("rvq_rest", -1, rest)
            x = x + torch.matmul(rest, w["quantizer.rvq_rest.output_proj"].t())
        return x

    # -- transformer -------------------------------------------------------
    def attention(self, l: int, y: torch.Tensor, offset: int = 0) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        B, T, D = y.shape
        H, hd = cfg.num_heads, cfg.head_dim
        qkv = torch.matmul(y, w[f"layers.{l}.self_attn.in_proj_weight"].t())  # [B, T, 3D]
        if offset == 0:
            # One launch splits the packed projection into head-major [B, H, T, hd]
            # Q and K (rotated, rope_i) and V: the layouts both attention GEMMs take
            # as they are, where the narrow / transpose views below cost a
            # contiguous copy of each. (A T-slot ring written from position 0 is
            # the sequence in order.)
            k = torch.empty((B, H, T, hd), dtype=qkv.dtype, device=qkv.device)
            v = torch.empty_like(k)
            q = xn.kv_append_rope(qkv, H, self.cos, self.sin, k, v, 0)
            scores = torch.matmul(q, k.transpose(2, 3))  # [B, H, T, T]
            probs = xn.attn_softmax(scores, self.scale, offset)
            ctx = torch.matmul(probs, v)  # [B, H, T, hd]
            for name, t in (("qkv", qkv), ("q", q), ("k", k), ("v", v), ("scores", scores), ("probs", probs)):
                self._rec(name, l, t)
        else:
            q, k = xn.rope_qk_packed(qkv, H, self.cos, self.sin, offset, interleaved=True)  # [B, T, H, hd]
            v = qkv[..., 2 * D:].view(B, T, H, hd)
            scores = torch.matmul(q.transpose(1, 2), k.permute(0, 2, 3, 1))  # [B, H, T, T]
            probs = xn.attn_softmax(scores, self.scale, offset)
            ctx = torch.matmul(probs, v.transpose(1, 2))  # [B, H, T, hd]
        return torch.matmul(ctx.transpose(1, 2).reshape(B, T, D), w[f"layers.{l}.self_attn.out_proj.weight"].t())

    def mlp(self, l: int, y: torch.Tensor) -> torch.Tensor:
        w = self.w
        h = torch.matmul(y, w[f"layers.{l}.linear1.weight"].t())
        self._rec("h_pre", l, h)
        xn.unary_(h, h, "gelu_erf")
        self._rec("h", l, h)
        return torch.matmul(h, w[f"layers.{l}.linear2.weight"].t())

    def transformer(self, x: torch.Tensor, offset: int = 0) -> torch.Tensor:
        """StreamingTransformer::forward over [B, T, D] with the norm / residual
        chain fused across layer boundaries."""
        cfg, w = self.cfg, self.w
        eps = cfg.eps
        resid = x
        y = xn.layer_norm(resid, w["layers.0.norm1.weight"], w["layers.0.norm1.bias"], eps)
        self._rec("x", 0, resid)
        self._rec("y", 0, y)
        for l in range(cfg.num_layers):
            p = f"layers.{l}."
            attn = self.attention(l, y, offset)
            # xs = xs + ls1 * attn ; norm2(xs)
            y2, resid = xn.layer_norm_residual(resid, attn, w[p + "norm2.weight"], w[p + "norm2.bias"], eps,
                                               layer_scale=w[p + "layer_scale_1.scale"])
            for name, t in (("attn", attn), ("y2", y2), ("resid_mid", resid)):
                self._rec(name, l, t)
            m = self.mlp(l, y2)
            self._rec("m", l, m)
            if l + 1 < cfg.num_layers:
                # xs = xs + ls2 * mlp ; next layer's norm1(xs)
                q = f"layers.{l + 1}."
                y, resid = xn.layer_norm_residual(resid, m, w[q + "norm1.weight"], w[q + "norm1.bias"], eps,
                                                  layer_scale=w[p + "layer_scale_2.scale"])
                self._rec("y", l + 1, y)
            else:
                resid = xn.residual_add(resid, m, w[p + "layer_scale_2.scale"])
            self._rec("resid", l, resid)
        return resid

    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n_q, T] -> decoder-transformer output [B, T, D]."""
        return self.transformer(self.rvq_decode(codes))


class StreamingDecoderChain:
    """The decoder transformer in streaming mode: each step takes t new frames
    [B, t, D] and attends to the last `context` positions through per-layer
    ring-buffer KV caches, as StreamingTransformer::forward with
    MimiStreamingMultiheadAttention does step by step
    (pocket_tts/src/mimi_transformer.rs:114-145, 234-266; mimi.rs:1317-1445).

    Per layer and step: fused LayerNorm (+ LayerScale + residual from the
    previous block), QKV GEMM, xn_decode_attention_step (split + rope_i on q
    and k + cache write, no cat / trim copies, then scores, scale, mask,
    softmax and the weighted sum of V, all in one launch), output GEMM, fused
    LayerNorm + residual, MLP (GEMM, GELU(erf) or SiLU in place, GEMM).

    The position counter lives in device memory, so `capture(t)` records one
    CUDA graph for a whole step (all layers + the position advance) that
    `step_graph` replays for every step."""

    def __init__(self, cfg: MimiChainConfig, weights: dict[str, torch.Tensor], cos: torch.Tensor,
                 sin: torch.Tensor, batch: int, *, act: str = "gelu_erf", mask: str = "absolute",
                 context: int | None = None):
        if act not in ("gelu_erf", "silu"):
            raise ValueError(f"unknown activation {act!r}")
        self.cfg, self.w, self.cos, self.sin = cfg, weights, cos, sin
        self.act, self.mask, self.batch = act, mask, batch
        self.context = int(context if context is not None else cfg.context)
        dtype = weights["layers.0.norm1.weight"].dtype
        dev = weights["layers.0.norm1.weight"].device
        H, hd = cfg.num_heads, cfg.head_dim
        self.scale = float(torch.tensor(1.0 / math.sqrt(hd), dtype=torch.float32).to(dtype).float())
        self.k = [torch.zeros((batch, H, self.context, hd), dtype=dtype, device=dev) for _ in range(cfg.num_layers)]
        self.v = [torch.zeros_like(k) for k in self.k]
        self.total = 0
        self.total_dev = torch.zeros(1, dtype=torch.int64, device=dev)
        self.graph = None
        # As MimiDecoderChain.trace (eager steps only; None while capturing).
        self.trace: list | None = None

    def _rec(self, name: str, layer: int, t: torch.Tensor) -> None:
        if self.trace is not None:
            self.trace.append((name, layer, t.detach().clone()))

    def reset(self) -> None:
        """Forget the stream (the caches' contents are overwritten as it refills)."""
        self.total = 0
        self.total_dev.zero_()

    def _layers(self, x: torch.Tensor, total: int | None, total_dev: torch.Tensor | None) -> torch.Tensor:
        cfg, w, eps = self.cfg, self.w, self.cfg.eps
        H = cfg.num_heads
        resid = x
        y = xn.layer_norm(resid, w["layers.0.norm1.weight"], w["layers.0.norm1.bias"], eps)
        self._rec("x", 0, resid)
        self._rec("y", 0, y)
        for l in range(cfg.num_layers):
            p = f"layers.{l}."
            qkv = torch.matmul(y, w[p + "self_attn.in_proj_weight"].t())
            a = xn.decode_attention_step(qkv, H, self.cos, self.sin, self.k[l], self.v[l], total, self.context,
                                         self.scale, interleaved=True, mask=self.mask, total_dev=total_dev)
            attn = torch.matmul(a, w[p + "self_attn.out_proj.weight"].t())
            y2, resid = xn.layer_norm_residual(resid, attn, w[p + "norm2.weight"], w[p + "norm2.bias"], eps,
                                               layer_scale=w[p + "layer_scale_1.scale"])
            h = torch.matmul(y2, w[p + "linear1.weight"].t())
            self._rec("h_pre", l, h)
            xn.unary_(h, h, self.act)
            m = torch.matmul(h, w[p + "linear2.weight"].t())
            for name, t in (("qkv", qkv), ("a", a), ("attn", attn), ("y2", y2), ("resid_mid", resid), ("h", h),
                            ("m", m)):
                self._rec(name, l, t)
            if l + 1 < cfg.num_layers:
                q_ = f"layers.{l + 1}."
                y, resid = xn.layer_norm_residual(resid, m, w[q_ + "norm1.weight"], w[q_ + "norm1.bias"], eps,
                                                  layer_scale=w[p + "layer_scale_2.scale"])
                self._rec("y", l + 1, y)
            else:
                resid = xn.residual_add(resid, m, w[p + "layer_scale_2.scale"])
            self._rec("resid", l, resid)
        return resid

    def _frames(self, x: torch.Tensor) -> int:
        """New positions in a step input (x [B, t, D])."""
        return x.shape[1]

    def _static_input(self, t: int) -> torch.Tensor:
        """The graph's input buffer for steps of t frames."""
        return torch.zeros((self.batch, t, self.cfg.d_model), dtype=self.k[0].dtype, device=self.total_dev.device)

    def step(self, x: torch.Tensor) -> torch.Tensor:
        """One eager step on x [B, t, D] with the host-side position."""
        out = self._layers(x, self.total, None)
        self.total += self._frames(x)
        self.total_dev.fill_(self.total)
        return out

    def capture(self, t: int = 1) -> None:
        """Records one step of t frames (reading the device position) as a CUDA graph."""
        dev = self.total_dev.device
        self.x_static = self._static_input(t)
        saved = self.total_dev.clone()
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):  # warm-up outside the graph (cuBLAS handles, workspaces)
            self._layers(self.x_static, None, self.total_dev)
        torch.cuda.current_stream(dev).wait_stream(stream)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.out_static = self._layers(self.x_static, None, self.total_dev)
            xn.position_advance(self.total_dev, t)
        self.total_dev.copy_(saved)
        self.graph_t = t

    def step_graph(self, x: torch.Tensor) -> torch.Tensor:
        """One step by graph replay; returns the graph's output buffer (valid
        until the next replay)."""
        self.x_static.copy_(x)
        self.graph.replay()
        self.total += self.graph_t
        return self.out_static


class MimiStreamingDecoder(StreamingDecoderChain):
    """Mimi::decode_step (mimi-rs/src/models/mimi.rs:2059-2071) on the fused
    ops, without its conv stages (the transposed-conv upsample and the SEANet
    decoder): each step takes the codes of t frames [B, n_q, t] (int64),
    decodes them with the two RVQ gather-sums and their 1x1 projections
    (SplitResidualVectorQuantizer::decode, :1858-1868), and runs one step of
    the decoder transformer (Transformer::step -> StreamingTransformer::forward,
    :1560-1571, 1476-1483) with mimi-rs's position bookkeeping: every layer's
    offset is the layer-0 cache's length before the step, min(total,
    context), used as the rope_i position and the causal-mask offset; caches
    keep the last `context` (250) positions as ring buffers. GELU(erf) MLP.
    `capture(t)` records the whole step (RVQ + all layers + the position
    advance) as one CUDA graph over a static codes buffer."""

    def __init__(self, cfg: MimiChainConfig, weights: dict[str, torch.Tensor], cos: torch.Tensor,
                 sin: torch.Tensor, batch: int, context: int | None = None):
        super().__init__(cfg, weights, cos, sin, batch, act="gelu_erf", mask="cache_len", context=context)
        self.rvq = MimiDecoderChain(cfg, weights, cos, sin)

    def _layers(self, codes: torch.Tensor, total: int | None, total_dev: torch.Tensor | None) -> torch.Tensor:
        self.rvq.trace = self.trace
        x = self.rvq.rvq_decode(codes)
        self.rvq.trace = None
        return super()._layers(x, total, total_dev)

    def _frames(self, codes: torch.Tensor) -> int:
        return codes.shape[2]

    def _static_input(self, t: int) -> torch.Tensor:
        return torch.zeros((self.batch, self.cfg.n_q, t), dtype=torch.int64, device=self.total_dev.device)
