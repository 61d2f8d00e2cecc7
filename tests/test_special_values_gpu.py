"""Non-finite and extreme inputs through the fused ops, against the oracle:
rows holding +-inf or NaN, and bf16 rows whose values are finite but large
enough that the f32 sum of squares overflows (RMSNorm's divisor becomes inf,
so the reference's x / m is +-0). The results must follow the reference's
IEEE arithmetic element for element: the same non-finite pattern, and the
same values elsewhere within the usual tolerance."""
import numpy as np
import pytest
import torch

from helpers import (assert_close, from_device, layer_norm_abs_bound, randn, rng, storage_to_f32, to_device,
                     to_storage)

pytestmark = pytest.mark.gpu


def _rows(dtype, cols):
    r = rng(cols)
    x = randn(r, (8, cols))
    x[1, 3] = np.inf
    x[2, 5] = -np.inf
    x[3, 7] = np.nan
    x[4, :] = 3.0e19  # finite; squares overflow f32 (sum of squares = inf)
    x[4, ::3] = -2.0e20
    x[5, :] = 0.0
    x[5, ::2] = -0.0  # signed zeros: x / m keeps the sign of x
    x[6, 0] = 1.0e30
    return to_storage(x, dtype)


def _same_nonfinite(got, ref, dtype, extra=None):
    g, r = storage_to_f32(got, dtype), storage_to_f32(ref, dtype)
    assert np.array_equal(np.isnan(g), np.isnan(r)), "NaN pattern differs"
    assert np.array_equal(np.isinf(g), np.isinf(r)), "inf pattern differs"
    assert np.array_equal(g[np.isinf(g)], r[np.isinf(r)]), "inf signs differ"
    fin = np.isfinite(r)
    if extra is not None:
        return got[fin], ref[fin], np.nan_to_num(extra[fin], nan=0.0, posinf=0.0)
    return got[fin], ref[fin]


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("cols", [37, 64, 1000])
def test_norms_and_softmax_special_values(oracle, xn, cuda, dtype, cols):
    x = _rows(dtype, cols)
    w = to_storage(randn(rng(1), cols, 0.02, 1.0), dtype)
    b = to_storage(randn(rng(2), cols, 0.1), dtype)
    X, W, B = (to_device(a, dtype, cuda) for a in (x, w, b))
    # LayerNorm's cancellation allowance (helpers.layer_norm_abs_bound), per row.
    with np.errstate(all="ignore"):
        ln_allow = layer_norm_abs_bound(storage_to_f32(x, dtype), storage_to_f32(w, dtype), 1e-5)
    for got, ref, what, allow in [
        (xn.rms_norm(X, W, 1e-5), oracle.rms_norm(x, w, 1e-5, dtype), "rms_norm", None),
        (xn.layer_norm(X, W, B, 1e-5), oracle.layer_norm(x, w, b, 1e-5, dtype), "layer_norm", ln_allow),
        (xn.softmax(X), oracle.softmax(x, dtype), "softmax", None),
    ]:
        full = from_device(got, dtype)
        g, r, e = _same_nonfinite(full, ref, dtype, np.zeros(ref.shape) if allow is None else allow)
        if g.size:
            assert_close(g, r, dtype, f"{what} finite part", extra_abs=e)
        # The row of signed zeros, bit for bit (+0 and -0 differ in storage).
        assert np.array_equal(full[5].view(np.uint32 if dtype == "f32" else np.uint16),
                              ref[5].view(np.uint32 if dtype == "f32" else np.uint16)), f"{what}: signed zeros"


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_activations_special_values(oracle, xn, cuda, dtype):
    x = to_storage(np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 88.0, -88.0, 1e30, -1e30], np.float32), dtype)
    X = to_device(x, dtype, cuda)
    for op in ("silu", "gelu_erf"):
        g, r = _same_nonfinite(from_device(getattr(xn, op)(X), dtype), oracle.unary(x, op, dtype), dtype)
        assert np.array_equal(g, r) or dtype == "f32", f"{op}"
        if dtype == "f32":
            assert_close(g, r, dtype, op)


# Widths that reach each softmax kernel with a causal mask: the scalar/pair
# rows (37), the window (250), the register pipe (1024, 1536; f32 4096), the
# shared-memory-staged rows (16-bit 4096, f32 12000), the cluster (16-bit
# 40000, f32 20000) and the loop kernel (16-bit 140000).
CAUSAL_WIDTHS = {"f32": [37, 250, 1024, 1536, 4096, 12000, 20000],
                 "bf16": [37, 250, 1024, 1536, 4096, 40000, 140000],
                 "f16": [37, 250, 1024, 4096, 40000]}


@pytest.mark.parametrize("dtype,cols", [(d, c) for d, cs in CAUSAL_WIDTHS.items() for c in cs])
def test_causal_softmax_special_values(oracle, xn, cuda, dtype, cols):
    """Causal rows holding +inf, NaN or only -inf among their live columns:
    the reference masks with -inf and then takes the softmax, so such a row's
    sum is NaN and every output of the row is NaN, the masked columns'
    0 / NaN included. +inf or NaN in masked columns is never read. The offset
    leaves most of each row masked, which selects the kernels' masked-vector
    skipping."""
    t1, offset = 8, cols // 4
    x = randn(rng(cols + 1), (1, t1, cols))
    x[0, 0, 0] = np.inf  # live
    x[0, 1, 1] = np.nan  # live
    x[0, 2, :] = -np.inf  # every live entry -inf
    x[0, 3, 2] = -np.inf  # one live entry -inf: an ordinary row
    x[0, 5, offset + 6:] = np.inf  # masked columns only
    x[0, 6, offset + 7:] = np.nan  # masked columns only
    x = to_storage(x, dtype)
    ref = oracle.softmax_causal(x, offset, dtype)
    got = from_device(xn.softmax_causal(to_device(x, dtype, cuda), offset), dtype)
    g, r = _same_nonfinite(got, ref, dtype)
    assert np.isnan(storage_to_f32(ref, dtype)[0, :3]).all()
    assert_close(g, r, dtype, f"softmax_causal {dtype} special values {cols}")


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_special_values(oracle, xn, cuda, dtype, interleaved):
    """RoPE on rows holding +-inf, NaN and values whose products overflow:
    each product and sum rounds to T as the reference's T arithmetic does
    (cpu_backend.rs:359-422), so the results match bit for bit, inf signs
    included; NaN positions match (their payloads are not compared)."""
    b, h, t, d, max_pos = 1, 3, 6, 16, 8
    x = randn(rng(d + t), (b, h, t, d))
    x[0, 0, 1, 2] = np.inf
    x[0, 0, 2, 9] = -np.inf
    x[0, 1, 3, 0] = np.nan
    x[0, 1, 4, :] = 6.0e4 if dtype == "f16" else 3.0e38  # products near the top of the range
    x[0, 2, 5, :] = -0.0
    x = to_storage(x, dtype)
    cos, sin = oracle.rope_tables(d, max_pos, 10000.0, dtype, "mimi")
    ref = oracle.rope(x, cos, sin, 2, dtype, interleaved=interleaved)
    f = xn.rope_i if interleaved else xn.rope
    got = from_device(f(to_device(x, dtype, cuda), to_device(cos, dtype, cuda), to_device(sin, dtype, cuda), 2),
                      dtype)
    g, r = storage_to_f32(got, dtype), storage_to_f32(ref, dtype)
    assert np.array_equal(np.isnan(g), np.isnan(r)), "NaN pattern differs"
    keep = ~np.isnan(r)
    assert np.array_equal(got[keep], ref[keep]), "non-NaN outputs differ"


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("cols", [64, 250, 1024])
def test_residual_norms_special_values(oracle, xn, cuda, dtype, cols):
    """The fused residual prologue h = T(x + T(branch * ls)) with +-inf, NaN
    and cancelling infinities in x or the branch: h bit for bit outside NaN
    positions (which match), then both norms of h with the same non-finite
    pattern as the reference."""
    r = rng(cols + 3)
    x = randn(r, (6, cols))
    br = randn(r, (6, cols))
    x[0, 1], br[0, 1] = np.inf, -np.inf  # inf + (-inf) = NaN
    x[1, 2] = np.nan
    br[2, 3] = np.inf
    x[3, :], br[3, :] = 1.0, -1.0  # exact cancellation: h = +0 everywhere (up to ls)
    x, br = to_storage(x, dtype), to_storage(br, dtype)
    ls = to_storage(r.uniform(0.5, 1.0, cols).astype(np.float32), dtype)
    w = to_storage(randn(r, cols, 0.02, 1.0), dtype)
    b = to_storage(randn(r, cols, 0.1), dtype)
    X, BR, LS, W, B = (to_device(a, dtype, cuda) for a in (x, br, ls, w, b))
    for name, (y, h), (ry, rh) in [
        ("rms_norm_residual", xn.rms_norm_residual(X, BR, W, 1e-5, layer_scale=LS),
         oracle.rms_norm_residual(x, br, w, 1e-5, dtype, layer_scale=ls)),
        ("layer_norm_residual", xn.layer_norm_residual(X, BR, W, B, 1e-5, layer_scale=LS),
         oracle.layer_norm_residual(x, br, w, b, 1e-5, dtype, layer_scale=ls)),
    ]:
        gh = from_device(h, dtype)
        assert np.array_equal(np.isnan(storage_to_f32(gh, dtype)), np.isnan(storage_to_f32(rh, dtype))), name
        keep = ~np.isnan(storage_to_f32(rh, dtype))
        assert np.array_equal(gh[keep], rh[keep]), f"{name}: residual output differs"
        gy = from_device(y, dtype)
        _same_nonfinite(gy, ry, dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_gather_copies_every_bit_pattern(xn, cuda, dtype):
    """The embedding gather is a byte copy: NaN payloads, infinities, signed
    zeros and subnormals arrive unchanged."""
    width = 64
    if dtype == "f32":
        pats = np.array([0x7fc00001, 0xffc00123, 0x7f800000, 0xff800000, 0x80000000, 0x00000001, 0x807fffff],
                        dtype=np.uint32)
    else:
        pats = np.array([0x7e01, 0xfe77, 0x7c00, 0xfc00, 0x8000, 0x0001, 0x83ff] if dtype == "f16"
                        else [0x7fc1, 0xffa3, 0x7f80, 0xff80, 0x8000, 0x0001, 0x807f], dtype=np.uint16)
    table = np.resize(pats, (40, width)).astype(pats.dtype)
    table[np.arange(40), np.arange(40) % width] = pats[0]
    ids = np.array([39, 0, 7, 7, 21, 3], dtype=np.int64)
    store = table.view(np.float32) if dtype == "f32" else table
    got = from_device(xn.index_select(to_device(store, dtype, cuda), torch.from_numpy(ids).to(cuda), 0), dtype)
    assert np.array_equal(got.view(pats.dtype), table[ids])
