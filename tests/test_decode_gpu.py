"""GPU parity for the streaming-decode rows: the KV-cache append fused with
RoPE (bit-exact against the reference's split + rope_i + cat/trim cache) and
the decode attention (against the reference's matmul_t / scale / mask /
softmax / matmul sequence on the oracle), over multi-step streams that wrap
the ring buffer and trim the context (mimi.rs:1099-1153, 1317-1384;
pocket_tts/src/transformer.rs:16-145, mimi_transformer.rs:10-61)."""
import numpy as np
import pytest
import torch

from helpers import assert_close, attention_abs_bound, from_device, randn, rng, storage_to_f32, to_device, to_storage

pytestmark = pytest.mark.gpu


def _tables(oracle, d, max_pos, dtype):
    return oracle.rope_tables(d, max_pos, 10000.0, dtype, "mimi")


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("b,h,t,d,cap,total", [(2, 4, 1, 64, 16, 0), (2, 4, 3, 64, 16, 14), (1, 2, 5, 32, 8, 6),
                                               (3, 16, 1, 64, 256, 255), (1, 2, 2, 128, 4, 9), (2, 3, 2, 6, 4, 1)])
def test_kv_append_rope_exact(oracle, xn, cuda, dtype, interleaved, b, h, t, d, cap, total):
    """q_out, and the cache slots (total + i) % cap, equal the reference's
    rope_i / rope of the split projection at pos = total, bit for bit; every
    other cache slot is left untouched. d = 6 exercises the scalar path."""
    r = rng(b * 1000 + h * 100 + t * 10 + d + total)
    max_pos = total + t + 3
    cos, sin = _tables(oracle, d, max_pos, dtype)
    qkv = to_storage(randn(r, (b, t, 3 * h * d)), dtype)
    kc0 = to_storage(randn(r, (b, h, cap, d)), dtype)
    vc0 = to_storage(randn(r, (b, h, cap, d)), dtype)
    K, V = to_device(kc0, dtype, cuda), to_device(vc0, dtype, cuda)
    Q = xn.kv_append_rope(to_device(qkv, dtype, cuda), h, to_device(cos, dtype, cuda), to_device(sin, dtype, cuda),
                          K, V, total, interleaved=interleaved)
    q, k, v = oracle.split_qkv(qkv, h)
    q_ref = oracle.rope(q, cos, sin, total, dtype, interleaved=interleaved)
    k_ref = oracle.rope(k, cos, sin, total, dtype, interleaved=interleaved)
    assert np.array_equal(from_device(Q, dtype), q_ref)
    kc, vc = from_device(K, dtype), from_device(V, dtype)
    slots = [(total + i) % cap for i in range(t)]
    kc_ref, vc_ref = kc0.copy(), vc0.copy()
    for i, s in enumerate(slots):
        kc_ref[:, :, s] = k_ref[:, :, i]
        vc_ref[:, :, s] = v[:, :, i]
    assert np.array_equal(kc, kc_ref)
    assert np.array_equal(vc, vc_ref)


def _stream(oracle, xn, cuda, dtype, *, b, h, d, cap, context, steps, mask, seed, interleaved=True,
            use_total_dev=False):
    """Runs a stream of decode steps (t per step from `steps`) on the GPU and
    through the reference op sequence; yields (got, ref) per step."""
    r = rng(seed)
    max_pos = sum(steps) + 4
    cos, sin = _tables(oracle, d, max_pos, dtype)
    cos_d, sin_d = to_device(cos, dtype, cuda), to_device(sin, dtype, cuda)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    K = torch.zeros((b, h, cap, d), dtype=tdt, device=cuda)
    V = torch.zeros_like(K)
    scale = float(1.0 / np.sqrt(np.float32(d)))
    cache = oracle.KvCacheRef(context)
    total = 0
    total_dev = torch.zeros(1, dtype=torch.int64, device=cuda) if use_total_dev else None
    for t in steps:
        qkv = to_storage(randn(r, (b, t, 3 * h * d)), dtype)
        qkv_d = to_device(qkv, dtype, cuda)
        if use_total_dev:
            Q = xn.kv_append_rope(qkv_d, h, cos_d, sin_d, K, V, interleaved=interleaved, total_dev=total_dev)
            O = xn.attention_decode(Q, K, V, None, context, scale, mask=mask, total_dev=total_dev)
            xn.position_advance(total_dev, t)
        else:
            Q = xn.kv_append_rope(qkv_d, h, cos_d, sin_d, K, V, total, interleaved=interleaved)
            O = xn.attention_decode(Q, K, V, total, context, scale, mask=mask)
        q, k, v = oracle.split_qkv(qkv, h)
        q = oracle.rope(q, cos, sin, total, dtype, interleaved=interleaved)
        k = oracle.rope(k, cos, sin, total, dtype, interleaved=interleaved)
        kk, vv = cache.append(k, v)
        kv_len = kk.shape[2]
        mask_offset = kv_len - t if mask == "relative" else total
        ref = oracle.attention_step(q, kk, vv, scale, mask_offset, dtype).reshape(b, t, h * d)
        # The reference's probabilities, for the weighted sum's allowance.
        scores = oracle.scale(oracle.matmul(q, kk, dtype, trans_rhs=True), scale, dtype)
        probs = oracle.softmax(oracle.apply_causality_mask(scores, mask_offset, dtype), dtype)
        allow = attention_abs_bound(storage_to_f32(probs, dtype), storage_to_f32(vv, dtype)).reshape(b, t, h * d)
        yield from_device(O, dtype), ref, allow
        total += t


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("mask", ["relative", "absolute"])
@pytest.mark.parametrize("d", [32, 64, 128])
def test_attention_decode_stream(oracle, xn, cuda, dtype, mask, d):
    """Single-token steps and chunks, past the context so the cache trims and
    the ring wraps (cap 24 > context 20)."""
    steps = [3, 1, 1, 4, 1, 2, 1, 1, 5, 1, 1, 1, 2, 1]
    for n, (got, ref, allow) in enumerate(_stream(oracle, xn, cuda, dtype, b=2, h=3, d=d, cap=24, context=20,
                                                  steps=steps, mask=mask, seed=d)):
        assert_close(got, ref, dtype, f"attention_decode {dtype} d={d} step {n}", extra_abs=allow)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_attention_decode_config3_shapes(oracle, xn, cuda, dtype):
    """Benchmark config 3 shapes (B=16, 16 heads of 64) over the first steps and
    a step at a long context (t=1 per step, pos = step - 1)."""
    for n, (got, ref, allow) in enumerate(_stream(oracle, xn, cuda, dtype, b=16, h=16, d=64, cap=256, context=256,
                                                  steps=[1] * 6, mask="relative", seed=3)):
        assert_close(got, ref, dtype, f"attention_decode {dtype} config3 step {n}", extra_abs=allow)


def test_attention_decode_device_position_matches_host(oracle, xn, cuda):
    """Reading the position from device memory (graph-capturable) gives the
    same results as passing it from the host."""
    steps = [2, 1, 1, 3, 1, 1, 1]
    host = [g for g, _, _ in _stream(oracle, xn, cuda, "bf16", b=2, h=4, d=64, cap=8, context=6, steps=steps,
                                  mask="relative", seed=11)]
    dev = [g for g, _, _ in _stream(oracle, xn, cuda, "bf16", b=2, h=4, d=64, cap=8, context=6, steps=steps,
                                 mask="relative", seed=11, use_total_dev=True)]
    for a, c in zip(host, dev):
        assert np.array_equal(a, c)


def test_decode_step_cuda_graph(oracle, xn, cuda):
    """One captured graph (append + attention + position advance) replayed
    for every step gives the eager results."""
    b, h, d, cap, context, steps = 2, 4, 64, 16, 12, 20
    dt = torch.bfloat16
    r = torch.Generator(device="cpu").manual_seed(5)
    cos, sin = (to_device(a, "bf16", cuda) for a in _tables(oracle, d, 64, "bf16"))
    qkvs = [torch.randn((b, 1, 3 * h * d), generator=r).to(dt).to(cuda) for _ in range(steps)]
    scale = 0.125

    def run_eager():
        K = torch.zeros((b, h, cap, d), dtype=dt, device=cuda)
        V = torch.zeros_like(K)
        outs = []
        for s in range(steps):
            Q = xn.kv_append_rope(qkvs[s], h, cos, sin, K, V, s)
            outs.append(xn.attention_decode(Q, K, V, s, context, scale).clone())
        return outs

    eager = run_eager()
    K = torch.zeros((b, h, cap, d), dtype=dt, device=cuda)
    V = torch.zeros_like(K)
    total = torch.zeros(1, dtype=torch.int64, device=cuda)
    x_in = torch.empty_like(qkvs[0])
    q_buf = torch.empty((b, h, 1, d), dtype=dt, device=cuda)
    out = torch.empty((b, 1, h * d), dtype=dt, device=cuda)
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        x_in.copy_(qkvs[0])
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            xn.kv_append_rope(x_in, h, cos, sin, K, V, interleaved=True, total_dev=total, q_out=q_buf)
            xn.attention_decode(q_buf, K, V, None, context, scale, total_dev=total, out=out)
            xn.position_advance(total, 1)
    outs = []
    for s in range(steps):
        x_in.copy_(qkvs[s])
        g.replay()
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert int(total.item()) == steps
    for a, c in zip(eager, outs):
        assert torch.equal(a, c)


def test_kv_append_device_position_out_of_range(oracle, xn, cuda):
    """A device position past the cos/sin tables writes nothing and sets the
    error flag (the host checks host positions before launching)."""
    b, h, t, d, cap = 1, 2, 2, 64, 8
    cos, sin = (to_device(a, "f32", cuda) for a in _tables(oracle, d, 4, "f32"))
    K = torch.full((b, h, cap, d), 7.0, device=cuda)
    V = torch.full_like(K, 7.0)
    qkv = torch.randn((b, t, 3 * h * d), device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    total = torch.tensor([3], dtype=torch.int64, device=cuda)  # positions 3 (ok) and 4 (out of range)
    xn.kv_append_rope(qkv, h, cos, sin, K, V, total_dev=total, err_flag=err)
    assert int(err.item()) == 1
    assert torch.all(K[:, :, 4] == 7.0) and torch.all(V[:, :, 4] == 7.0)  # slot of position 4 untouched
    assert not torch.all(K[:, :, 3] == 7.0)  # position 3 written
    with pytest.raises(xn.XnError, match="out of range"):
        xn.kv_append_rope(qkv, h, cos, sin, K, V, 3)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("d", [32, 64, 128])
def test_fused_step_equals_two_launches(oracle, xn, cuda, dtype, interleaved, d):
    """xn_decode_attention_step gives the outputs and cache contents of
    xn_kv_append_rope + xn_attention_decode, bit for bit, over a stream with
    chunks, wrap and trim."""
    b, h, cap, context = 2, 3, 12, 10
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    cos, sin = (to_device(a, dtype, cuda) for a in _tables(oracle, d, 64, dtype))
    g = torch.Generator().manual_seed(d)
    K1 = torch.zeros((b, h, cap, d), dtype=tdt, device=cuda)
    V1, K2, V2 = torch.zeros_like(K1), torch.zeros_like(K1), torch.zeros_like(K1)
    total = 0
    for t in [3, 1, 2, 1, 1, 4, 1, 2, 1]:
        qkv = torch.randn((b, t, 3 * h * d), generator=g).to(tdt).to(cuda)
        for mask in ("relative", "absolute"):
            K1c, V1c, K2c, V2c = K1.clone(), V1.clone(), K2.clone(), V2.clone()
            q = xn.kv_append_rope(qkv, h, cos, sin, K1c, V1c, total, interleaved=interleaved)
            a = xn.attention_decode(q, K1c, V1c, total, context, 0.125, mask=mask)
            f = xn.decode_attention_step(qkv, h, cos, sin, K2c, V2c, total, context, 0.125,
                                         interleaved=interleaved, mask=mask)
            assert torch.equal(a, f)
            assert torch.equal(K1c, K2c) and torch.equal(V1c, V2c)
        xn.kv_append_rope(qkv, h, cos, sin, K1, V1, total, interleaved=interleaved)
        xn.decode_attention_step(qkv, h, cos, sin, K2, V2, total, context, 0.125, interleaved=interleaved)
        total += t
