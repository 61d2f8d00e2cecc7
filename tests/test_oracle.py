"""CPU tests of the oracle: it must reproduce every known-answer test the
reference holds for this path, and its f32 arithmetic must agree with float64
mathematics; its bf16 conversion must match torch's round-to-nearest-even."""
import numpy as np
import pytest
import torch

from helpers import randn, rng, storage_to_f32, to_storage
from known_answers import OracleRunner, load_cases, run_case


@pytest.mark.parametrize("case", load_cases(), ids=lambda c: c["name"])
def test_known_answers(oracle, case):
    run_case(case, OracleRunner(oracle))


def test_bf16_conversion_matches_torch(oracle):
    r = rng(1)
    x = np.concatenate([randn(r, 100000, 3.0), np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, -3.4e38, np.inf, -np.inf],
                                                          dtype=np.float32)])
    ref = to_storage(x, "bf16")
    L = oracle.lib()
    got = np.array([L.xo_f32_to_bf16(float(v)) for v in x[:2000]] + [L.xo_f32_to_bf16(float(v)) for v in x[-8:]],
                   dtype=np.uint16)
    assert np.array_equal(got, np.concatenate([ref[:2000], ref[-8:]]))
    # Ties to even: 1 + 2^-8 is exactly between two bf16 values.
    assert L.xo_f32_to_bf16(1.0 + 2.0 ** -8) == 0x3F80
    assert L.xo_f32_to_bf16(1.0 + 3 * 2.0 ** -8) == 0x3F82


def test_rms_norm_f32_vs_float64(oracle):
    r = rng(2)
    x, a = randn(r, (64, 1000)), randn(r, 1000, 0.02, 1.0)
    got = oracle.rms_norm(x, a, 1e-5, "f32").astype(np.float64)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt((xd ** 2).mean(-1, keepdims=True) + 1e-5) * a
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)) < 1e-5


def test_layer_norm_f32_vs_float64(oracle):
    r = rng(3)
    x, w, b = randn(r, (64, 512), 2.0, 1.0), randn(r, 512, 0.02, 1.0), randn(r, 512, 0.1)
    for rm in (True, False):
        got = oracle.layer_norm(x, w, b, 1e-5, "f32", remove_mean=rm).astype(np.float64)
        xd = x.astype(np.float64)
        mean = xd.mean(-1, keepdims=True)
        var = ((xd - mean) ** 2).mean(-1, keepdims=True)
        ref = ((xd - mean) if rm else xd) / np.sqrt(var + 1e-5) * w + b
        assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-2)) < 1e-4


def test_softmax_causal_composite(oracle):
    r = rng(4)
    x = randn(r, (2, 3, 5, 7), 2.0)
    y = oracle.softmax_causal(x, 1, "f32")
    xd = x.astype(np.float64)
    i = np.arange(5)[:, None]
    j = np.arange(7)[None, :]
    xd = np.where(j > i + 1, -np.inf, xd)
    e = np.exp(xd - xd.max(-1, keepdims=True))
    ref = e / e.sum(-1, keepdims=True)
    assert np.allclose(y, ref, atol=1e-6)
    assert np.all(y[..., 0, 2:] == 0)


def test_rope_matches_complex_rotation(oracle):
    r = rng(5)
    b, h, t, d = 2, 3, 7, 16
    x = randn(r, (b, h, t, d))
    cos, sin = oracle.rope_tables(d, 32, 10000.0, "f32", "llama")
    y = oracle.rope(x, cos, sin, 5, "f32")
    c, s = cos[5:5 + t][None, None], sin[5:5 + t][None, None]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    ref = np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], -1)
    assert np.allclose(y, ref, atol=1e-6)
    yi = oracle.rope(x, cos, sin, 5, "f32", interleaved=True)
    xe, xo = x[..., 0::2], x[..., 1::2]
    refi = np.stack([xe * c - xo * s, xe * s + xo * c], -1).reshape(x.shape)
    assert np.allclose(yi, refi, atol=1e-6)


def test_rope_tables_variants_agree(oracle):
    # i / half_dim and 2i / head_dim are the same f32 quotient.
    cm, sm = oracle.rope_tables(128, 64, 500000.0, "f32", "mimi")
    cl, sl = oracle.rope_tables(128, 64, 500000.0, "f32", "llama")
    assert np.array_equal(cm, cl) and np.array_equal(sm, sl)


def test_bf16_chain_rounds_each_op(oracle):
    """rope in bf16 rounds each product and sum (half's bf16 arithmetic)."""
    x = to_storage(np.array([1.0078125, 3.0], dtype=np.float32), "bf16").reshape(1, 1, 1, 2)
    cos = to_storage(np.array([[1.0078125]], dtype=np.float32), "bf16")
    sin = to_storage(np.array([[0.0]], dtype=np.float32), "bf16")
    y = storage_to_f32(oracle.rope(x, cos, sin, 0, "bf16"), "bf16")
    # 1.0078125^2 = 1.01568603515625 -> bf16 1.015625
    assert y.ravel()[0] == np.float32(1.015625)


def test_gelu_and_silu_f32_vs_float64(oracle):
    from math import erf

    r = rng(6)
    x = randn(r, 4096, 3.0)
    g = oracle.unary(x, "gelu_erf", "f32").astype(np.float64)
    ref = np.array([v * 0.5 * (1 + erf(v / np.sqrt(2))) for v in x.astype(np.float64)])
    # The reference formula cancels in 1 + erf(x/sqrt2) for x << 0, so the f32
    # result carries an absolute error of a few 1e-7 there.
    assert np.all(np.abs(g - ref) <= 1e-5 * np.abs(ref) + 1e-6)
    s = oracle.unary(x, "silu", "f32").astype(np.float64)
    xd = x.astype(np.float64)
    refs = xd / (1 + np.exp(-xd))
    assert np.max(np.abs(s - refs) / np.maximum(np.abs(refs), 1e-3)) < 1e-5


def test_rvq_composite_matches_numpy(oracle):
    r = rng(7)
    q, bins, dim, b, t = 4, 64, 16, 2, 9
    books = [randn(r, (bins, dim)) for _ in range(q)]
    codes = r.integers(0, bins, size=(b, q, t), dtype=np.int64)
    got = oracle.rvq_decode(books, codes, "f32", "bct")
    ref = np.zeros((b, t, dim), dtype=np.float32)
    for i in range(q):
        ref = ref + books[i][codes[:, i, :]] if i else books[i][codes[:, i, :]]
    assert np.array_equal(got, np.swapaxes(ref, 1, 2))


def test_thread_count_does_not_change_results(oracle):
    r = rng(8)
    x, a = randn(r, (257, 333)), randn(r, 333, 0.02, 1.0)
    n = oracle.get_num_threads()
    try:
        oracle.set_num_threads(1)
        y1 = oracle.rms_norm(x, a, 1e-5, "f32")
        oracle.set_num_threads(max(2, n))
        y2 = oracle.rms_norm(x, a, 1e-5, "f32")
    finally:
        oracle.set_num_threads(n)
    assert np.array_equal(y1, y2)
    assert torch.get_num_threads() >= 1


def test_matmul_oracle_matches_float64(oracle):
    """xo_matmul (the reference's gemm contract: f32 accumulation, one T
    rounding) against a float64 product, f32 and bf16, plain and transposed."""
    r = rng(9)
    a, bt = randn(r, (3, 5, 64)), randn(r, (3, 7, 64))
    exact = np.einsum("bmk,bnk->bmn", a.astype(np.float64), bt.astype(np.float64))
    got = oracle.matmul(a, bt, "f32", trans_rhs=True)
    assert np.max(np.abs(got - exact)) <= 64 * 2.0 ** -24 * np.max(np.abs(a)) * np.max(np.abs(bt)) * 8
    got2 = oracle.matmul(a, np.ascontiguousarray(np.swapaxes(bt, 1, 2)), "f32")
    assert np.array_equal(got, got2)
    ah, bh = to_storage(a, "bf16"), to_storage(bt, "bf16")
    gh = storage_to_f32(oracle.matmul(ah, bh, "bf16", trans_rhs=True), "bf16")
    ex = np.einsum("bmk,bnk->bmn", storage_to_f32(ah, "bf16").astype(np.float64),
                   storage_to_f32(bh, "bf16").astype(np.float64))
    assert np.all(np.abs(gh - ex) <= np.abs(ex) * 2.0 ** -8 + 1e-6)


def test_kv_cache_ref_is_cat_then_trim(oracle):
    """KvCacheRef keeps the last max_seq_len positions in order
    (mimi.rs:1122-1153)."""
    cache = oracle.KvCacheRef(5)
    seen = []
    for step, t in enumerate([2, 1, 3, 1, 4]):
        k = np.arange(t, dtype=np.float32).reshape(1, 1, t, 1) + 10 * step
        kk, vv = cache.append(k, k + 0.5)
        seen.extend(k.ravel().tolist())
        assert kk.ravel().tolist() == seen[-5:]
        assert np.array_equal(vv, kk + 0.5)


def test_attention_step_rows_are_distributions(oracle):
    """The reference attention sequence on f32: with v = identity rows the
    output rows are the softmax probabilities (non-negative, summing to 1,
    zero past the causal limit)."""
    r = rng(10)
    b, h, t, kv, d = 1, 2, 3, 6, 6
    q, k = randn(r, (b, h, t, d)), randn(r, (b, h, kv, d))
    v = np.broadcast_to(np.eye(kv, d, dtype=np.float32), (b, h, kv, d)).copy()
    out = oracle.attention_step(q, k, v, 0.5, kv - t, "f32")  # [b, t, h, d]
    p = np.transpose(out, (0, 2, 1, 3))
    assert np.all(p >= 0)
    assert np.allclose(p.sum(-1), 1.0, atol=1e-6)
    for i in range(t):
        assert np.all(p[:, :, i, kv - t + i + 1:] == 0)
