"""End-to-end parity of the Mimi decoder chain (benchmark config 2 shapes:
batch 4, 250 frames, d_model 512, 8 heads of 64, 8 layers, FFN 2048, 8
codebooks of 2048 x 256) against the reference op sequence on the CPU oracle,
with seeded synthetic weights (no checkpoint is available offline)."""
import numpy as np
import pytest
import torch

from helpers import from_device
from mimi_oracle import chain_ref

pytestmark = pytest.mark.gpu


def _setup(dtype_name, cfg_kwargs, B, T, seed=0):
    import mimi_chain as mc

    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dtype_name]
    cfg = mc.MimiChainConfig(**cfg_kwargs)
    dev = torch.device("cuda:0")
    w = mc.synthetic_weights(cfg, tdt, dev, seed)
    cos, sin = mc.rope_tables(cfg, tdt, dev)
    chain = mc.MimiDecoderChain(cfg, w, cos, sin)
    g = torch.Generator().manual_seed(seed + 1)
    codes = torch.randint(0, cfg.bins, (B, cfg.n_q, T), generator=g, dtype=torch.int64)
    return mc, cfg, w, cos, sin, chain, codes, dev


def _np(w, dtype_name):
    return {k: from_device(v, dtype_name) for k, v in w.items()}


@pytest.mark.parametrize("dtype,tol", [("f32", 2e-4), ("bf16", 5e-2)])
def test_mimi_chain_matches_reference_sequence(oracle, xn, cuda, dtype, tol):
    """Full config-2 chain. f32: max |error| <= 2e-4 * rms(output); the GEMM
    libraries' summation orders differ (cuBLAS vs numpy), nothing else does.
    bf16: the same, at bf16 resolution (one-ulp GEMM differences propagate
    through 8 layers), checked as a relative RMS error."""
    mc, cfg, w, cos, sin, chain, codes, dev = _setup(dtype, {}, 4, 250)
    torch.backends.cuda.matmul.allow_tf32 = False
    got = from_device(chain.decode(codes.to(dev)), dtype)
    ref = chain_ref(oracle, cfg, _np(w, dtype), from_device(cos, dtype), from_device(sin, dtype), codes.numpy(),
                    dtype, chain.scale)
    from helpers import storage_to_f32

    g, r = storage_to_f32(got, dtype).astype(np.float64), storage_to_f32(ref, dtype).astype(np.float64)
    rms = np.sqrt(np.mean(r ** 2))
    if dtype == "f32":
        err = np.max(np.abs(g - r)) / rms
    else:
        err = np.sqrt(np.mean((g - r) ** 2)) / rms
    print(f"mimi chain {dtype}: error {err:.3e} of rms {rms:.3f}")
    assert err <= tol


def test_mimi_rvq_stage_exact(oracle, xn, cuda):
    """The RVQ gather-sums are bit-exact; only the projection GEMM differs."""
    mc, cfg, w, cos, sin, chain, codes, dev = _setup("f32", {}, 2, 37)
    books = [from_device(w[f"quantizer.codebook.{i}"], "f32") for i in range(cfg.n_q)]
    c = codes.numpy()
    ref_rest = oracle.rvq_decode(books[1:], np.ascontiguousarray(c[:, 1:]), "f32", "btd")
    got_rest = xn.rvq_decode_sum([w[f"quantizer.codebook.{i}"] for i in range(1, cfg.n_q)],
                                 codes[:, 1:].contiguous().to(dev), out_layout="btd")
    assert np.array_equal(from_device(got_rest, "f32"), ref_rest)


def test_mimi_chain_small_config_f32(oracle, xn, cuda):
    """A 2-layer, 4-head variant with ragged frame count."""
    kw = dict(d_model=64, num_heads=4, num_layers=2, dim_feedforward=128, n_q=3, bins=64, q_dim=32)
    mc, cfg, w, cos, sin, chain, codes, dev = _setup("f32", kw, 3, 17)
    torch.backends.cuda.matmul.allow_tf32 = False
    got = from_device(chain.decode(codes.to(dev)), "f32")
    ref = chain_ref(oracle, cfg, _np(w, "f32"), from_device(cos, "f32"), from_device(sin, "f32"), codes.numpy(),
                    "f32", chain.scale)
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= 2e-4 * rms


def _stream_setup(dtype_name, cfg_kwargs, B, seed=0, **chain_kw):
    import mimi_chain as mc

    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dtype_name]
    cfg = mc.MimiChainConfig(**cfg_kwargs)
    dev = torch.device("cuda:0")
    w = mc.synthetic_weights(cfg, tdt, dev, seed)
    cos, sin = mc.rope_tables(cfg, tdt, dev)
    chain = mc.StreamingDecoderChain(cfg, w, cos, sin, B, **chain_kw)
    return mc, cfg, w, cos, sin, chain, dev, tdt


def _rel_err(got, ref, dtype, how):
    from helpers import storage_to_f32

    g, r = storage_to_f32(got, dtype).astype(np.float64), storage_to_f32(ref, dtype).astype(np.float64)
    rms = np.sqrt(np.mean(r ** 2))
    return (np.max(np.abs(g - r)) if how == "max" else np.sqrt(np.mean((g - r) ** 2))) / rms


@pytest.mark.parametrize("mask", ["absolute", "relative"])
@pytest.mark.parametrize("act", ["gelu_erf", "silu"])
def test_streaming_chain_matches_reference_stream(oracle, xn, cuda, mask, act):
    """Small f32 config with chunked steps past the context (cache trims, ring
    wraps): every step's output against the reference streaming sequence."""
    from mimi_oracle import stream_ref

    torch.backends.cuda.matmul.allow_tf32 = False
    kw = dict(d_model=128, num_heads=4, num_layers=2, dim_feedforward=256)
    mc, cfg, w, cos, sin, chain, dev, tdt = _stream_setup("f32", kw, 3, act=act, mask=mask, context=6)
    g = torch.Generator().manual_seed(7)
    steps = [2, 1, 3, 1, 1, 2, 1]
    xs = [torch.randn((3, t, cfg.d_model), generator=g) for t in steps]
    got = [from_device(chain.step(x.to(dev)), "f32") for x in xs]
    ref = stream_ref(oracle, cfg, _np(w, "f32"), from_device(cos, "f32"), from_device(sin, "f32"),
                     [x.numpy() for x in xs], "f32", chain.scale, 6, act=act, mask=mask)
    for s, (a, b) in enumerate(zip(got, ref)):
        assert _rel_err(a, b, "f32", "max") <= 2e-4, f"step {s}"


@pytest.mark.parametrize("dtype,tol", [("f32", 2e-4), ("bf16", 5e-2)])
def test_streaming_chain_config3(oracle, xn, cuda, dtype, tol):
    """Benchmark config 3 shapes (B 16, D 1024, 16 heads of 64, 6 layers, MLP
    4096, SiLU) for the first steps, t = 1 per step."""
    from mimi_oracle import stream_ref

    torch.backends.cuda.matmul.allow_tf32 = False
    kw = dict(d_model=1024, num_heads=16, num_layers=6, dim_feedforward=4096)
    mc, cfg, w, cos, sin, chain, dev, tdt = _stream_setup(dtype, kw, 16, act="silu", context=256)
    g = torch.Generator().manual_seed(3)
    xs = [torch.randn((16, 1, 1024), generator=g).to(tdt) for _ in range(4)]
    got = [from_device(chain.step(x.to(dev)), dtype) for x in xs]
    ref = stream_ref(oracle, cfg, _np(w, dtype), from_device(cos, dtype), from_device(sin, dtype),
                     [from_device(x, dtype) for x in xs], dtype, chain.scale, 256, act="silu")
    for s, (a, b) in enumerate(zip(got, ref)):
        err = _rel_err(a, b, dtype, "max" if dtype == "f32" else "rms")
        assert err <= tol, f"step {s}: {err:.3e}"


def test_streaming_chain_graph_replay_matches_eager(xn, cuda):
    """One captured step graph replayed over 40 steps (past the context of 32)
    equals eager stepping bit for bit."""
    kw = dict(d_model=256, num_heads=4, num_layers=3, dim_feedforward=512)
    _, cfg, w, cos, sin, eager, dev, tdt = _stream_setup("bf16", kw, 4, context=32)
    import mimi_chain as mc

    graphed = mc.StreamingDecoderChain(cfg, w, cos, sin, 4, context=32)
    graphed.capture(1)
    g = torch.Generator().manual_seed(1)
    for s in range(40):
        x = torch.randn((4, 1, cfg.d_model), generator=g).to(tdt).to(dev)
        a = eager.step(x)
        b = graphed.step_graph(x)
        assert torch.equal(a, b), f"step {s}"
    assert int(graphed.total_dev.item()) == 40


# ---------------------------------------------------------------------------
# Teacher-forced chain parity: every fused op inside the chain against the
# oracle, fed the inputs the GPU chain gave it (tests/chain_check.py).
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_mimi_chain_teacher_forced(oracle, xn, cuda, dtype):
    """Config 2 (batch 4 x 250 frames, 8 layers): RVQ gather-sums and
    residual streams bit-exact; every LayerNorm, softmax and GELU output of
    all 8 layers within 1e-5 (f32) / 1 ulp (bf16) of the reference op on the
    same inputs."""
    from chain_check import check_whole_sequence, collect

    mc, cfg, w, cos, sin, chain, codes, dev = _setup(dtype, {}, 4, 250)
    chain.trace = []
    chain.decode(codes.to(dev))
    tr = collect(chain.trace, dtype)
    check_whole_sequence(oracle, cfg, _np(w, dtype), from_device(cos, dtype), from_device(sin, dtype), tr,
                         codes.numpy(), dtype, chain.scale)


def _stream_teacher_forced(oracle, chain, cfg, w, cos, sin, inputs, dtype, act, mask, what, codes=False):
    """Steps `chain` over `inputs`, checking every step's fused ops against the
    oracle fed the step's own inputs; returns the per-step outputs."""
    from chain_check import check_rvq, check_stream_step, collect

    wn, cn, sn = _np(w, dtype), from_device(cos, dtype), from_device(sin, dtype)
    caches = [oracle.KvCacheRef(chain.context) for _ in range(cfg.num_layers)]
    total, outs = 0, []
    for s, x in enumerate(inputs):
        chain.trace = []
        outs.append(from_device(chain.step(x), dtype))
        tr = collect(chain.trace, dtype)
        chain.trace = None
        if codes:
            check_rvq(oracle, cfg, wn, tr, x.cpu().numpy(), dtype)
        check_stream_step(oracle, cfg, wn, cn, sn, tr, caches, total, dtype, chain.scale, act, mask, f"{what} step {s}")
        total += chain._frames(x)
    return outs


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_streaming_chain_config3_teacher_forced(oracle, xn, cuda, dtype):
    """Config 3 (B 16, D 1024, 16 heads of 64, 6 layers, SiLU MLP), first
    steps: every fused op of every layer at the fused-op tolerance."""
    kw = dict(d_model=1024, num_heads=16, num_layers=6, dim_feedforward=4096)
    mc, cfg, w, cos, sin, chain, dev, tdt = _stream_setup(dtype, kw, 16, act="silu", context=256)
    g = torch.Generator().manual_seed(3)
    xs = [torch.randn((16, 1, 1024), generator=g).to(tdt).to(dev) for _ in range(4)]
    _stream_teacher_forced(oracle, chain, cfg, w, cos, sin, xs, dtype, "silu", "absolute", "config3")


@pytest.mark.parametrize("mask", ["absolute", "relative", "cache_len"])
def test_streaming_chain_teacher_forced_past_context(oracle, xn, cuda, mask):
    """A small f32 config streamed past its context of 6 with chunked steps
    (caches trim, rings wrap; "cache_len" rotates at the capped offset)."""
    kw = dict(d_model=128, num_heads=4, num_layers=2, dim_feedforward=256)
    mc, cfg, w, cos, sin, chain, dev, tdt = _stream_setup("f32", kw, 3, act="gelu_erf", mask=mask, context=6)
    g = torch.Generator().manual_seed(17)
    xs = [torch.randn((3, t, cfg.d_model), generator=g).to(dev) for t in [2, 1, 3, 1, 1, 2, 1, 4, 1]]
    _stream_teacher_forced(oracle, chain, cfg, w, cos, sin, xs, "f32", "gelu_erf", mask, f"past-context {mask}")


def _mimi_stream_setup(dtype, cfg_kwargs, B, context, seed=0):
    import mimi_chain as mc

    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dtype]
    cfg = mc.MimiChainConfig(**cfg_kwargs)
    dev = torch.device("cuda:0")
    w = mc.synthetic_weights(cfg, tdt, dev, seed)
    cos, sin = mc.rope_tables(cfg, tdt, dev)
    return cfg, w, cos, sin, mc.MimiStreamingDecoder(cfg, w, cos, sin, B, context=context), dev


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_mimi_streaming_decoder_teacher_forced(oracle, xn, cuda, dtype):
    """Mimi::decode_step at the Mimi transformer's shapes (D 512, 8 heads,
    8 layers, FFN 2048, 8 codebooks) with a context of 8 so a short stream
    passes it: per step the RVQ gather-sums (bit-exact) and every fused op of
    every layer at the fused-op tolerance; then the outputs end to end against
    the reference's stream (Mimi offsets: min(total, context))."""
    from mimi_oracle import stream_ref

    torch.backends.cuda.matmul.allow_tf32 = False
    B, context = 2, 8
    cfg, w, cos, sin, dec, dev = _mimi_stream_setup(dtype, {}, B, context, seed=5)
    g = torch.Generator().manual_seed(6)
    steps = [1, 1, 2, 1, 3, 1, 1, 1, 2, 1, 1]
    codes = [torch.randint(0, cfg.bins, (B, cfg.n_q, t), generator=g, dtype=torch.int64).to(dev) for t in steps]
    outs = _stream_teacher_forced(oracle, dec, cfg, w, cos, sin, codes, dtype, "gelu_erf", "cache_len",
                                  "mimi-stream", codes=True)
    ref = stream_ref(oracle, cfg, _np(w, dtype), from_device(cos, dtype), from_device(sin, dtype),
                     [c.cpu().numpy() for c in codes], dtype, dec.scale, context, act="gelu_erf", mask="cache_len",
                     codes=True)
    for s, (a, b) in enumerate(zip(outs, ref)):
        err = _rel_err(a, b, dtype, "max" if dtype == "f32" else "rms")
        assert err <= (2e-4 if dtype == "f32" else 5e-2), f"step {s}: {err:.3e}"


def test_mimi_streaming_decoder_graph_config2(oracle, xn, cuda):
    """Config 2's streaming form: batch 4, context 250, one frame per step for
    256 steps (past the context, where the offset stops at 250), one captured
    CUDA graph replayed per step, bit for bit equal to eager stepping (whose
    ops test_mimi_streaming_decoder_teacher_forced checks against the
    reference)."""
    cfg, w, cos, sin, eager, dev = _mimi_stream_setup("bf16", {}, 4, 250, seed=7)
    import mimi_chain as mc

    graphed = mc.MimiStreamingDecoder(cfg, w, cos, sin, 4, context=250)
    graphed.capture(1)
    g = torch.Generator().manual_seed(8)
    codes = [torch.randint(0, cfg.bins, (4, cfg.n_q, 1), generator=g, dtype=torch.int64) for _ in range(256)]
    for s, c in enumerate(codes):
        a = eager.step(c.to(dev))
        b = graphed.step_graph(c.to(dev))
        assert torch.equal(a, b), f"step {s}"
    assert int(graphed.total_dev.item()) == 256
