"""GPU parity: row softmax, the fused causal softmax and the stand-alone
causal mask against the oracle (cpu_backend.rs:647-689; the causal composite
is apply_causality_mask then softmax, llama.rs:201-202)."""
import numpy as np
import pytest

from helpers import F32_FLOOR, RECORDS, assert_close, from_device, randn, rng, sum_error_bound, to_device, to_storage

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "bf16", "f16"]


def assert_softmax_close(got, ref, dtype, cols, what):
    """assert_close, with the f32 bound widened for wide rows: y = e / sum, and
    the reference's sequential f32 row sum is itself only accurate to
    helpers.sum_error_bound(cols, sum) (4 * sqrt(n) * 2^-24 relative, 1.2e-5
    at n = 40000); the kernel's tree sum differs from it by that much, which
    moves every output of the row by the same relative amount. So f32 rows
    allow max(1e-5, 4 * sqrt(n) * 2^-24) of |ref| per element (floored at
    1e-3 * rms(ref), as assert_close). 16-bit outputs keep the 1-ulp bound."""
    bound = float(sum_error_bound(cols, 1.0))
    if dtype != "f32" or bound <= 1e-5:
        return assert_close(got, ref, dtype, what)
    g, e = got.astype(np.float64), ref.astype(np.float64)
    finite = np.isfinite(e)
    assert np.array_equal(np.isfinite(g), finite), f"{what}: non-finite pattern differs"
    floor = F32_FLOOR * np.sqrt(np.mean(e[finite] ** 2)) if finite.any() else 0.0
    rel = np.where(finite, np.abs(g - e) / np.maximum(np.maximum(np.abs(e), floor), 1e-300), 0.0)
    RECORDS.append({"what": what, "dtype": dtype, "n": int(e.size), "max_rel": float(rel.max()), "bound": bound})
    assert rel.max() <= bound, f"{what}: max relative error {rel.max():.3e} > {bound:.3e}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(1, 1), (2, 3), (5, 7), (64, 64), (300, 250), (64, 512), (8, 1000),
                                       (4, 4096), (3, 16384), (2, 20000), (7, 2), (33, 10), (20000, 250),
                                       (9, 1002), (3, 8194), (3, 65536),
                                       # staged kernel with 5 / 6 vectors per thread (16-bit 2560, 3072, 5120)
                                       (300, 2560), (300, 3072), (300, 5120),
                                       # pipe kernel, whole-vector rows with 3, 5 or 6 accesses per thread
                                       (300, 768), (300, 1536), (300, 1280), (64, 4100)])
def test_softmax(oracle, xn, cuda, dtype, rows, cols):
    r = rng(rows * 13 + cols)
    x = to_storage(randn(r, (rows, cols), 2.0), dtype)
    ref = oracle.softmax(x, dtype)
    Y = xn.softmax(to_device(x, dtype, cuda))
    assert_softmax_close(from_device(Y, dtype), ref, dtype, cols, f"softmax {dtype} {rows}x{cols}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(600, 40000), (2, 131072), (5, 100000)])
def test_softmax_widest_rows(oracle, xn, cuda, dtype, rows, cols):
    """Rows of tens of thousands of columns: the cluster kernel (up to 256 KB
    per row) and, past it, the three-pass kernel (f32 bound widened with
    sqrt(n), see assert_softmax_close)."""
    r = rng(rows + cols)
    x = to_storage(randn(r, (rows, cols), 2.0), dtype)
    ref = oracle.softmax(x, dtype)
    X = to_device(x, dtype, cuda)
    Y = xn.softmax(X)
    assert_softmax_close(from_device(Y, dtype), ref, dtype, cols, f"softmax {dtype} {rows}x{cols}")
    xn.softmax_(X, X)  # in place (dst == src), bit for bit the same
    assert np.array_equal(from_device(X, dtype), from_device(Y, dtype))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,offset", [((1, 16, 512, 512), 0), ((2, 3, 5, 7), 0), ((2, 3, 5, 7), 2),
                                          ((16, 16, 1, 200), 199), ((4, 8, 64, 96), 32), ((3, 9, 40), 0),
                                          ((1, 2, 3, 17000), 16990), ((4, 8, 250, 250), 0),
                                          ((2, 8, 37, 250), 100), ((3, 2, 11, 6), 1), ((1, 1, 4, 70000), 69990),
                                          ((1, 2, 3, 40000), 100)])
def test_softmax_causal(oracle, xn, cuda, dtype, shape, offset):
    r = rng(sum(shape) + offset)
    x = to_storage(randn(r, shape, 2.0), dtype)
    ref = oracle.softmax_causal(x, offset, dtype)
    Y = from_device(xn.softmax_causal(to_device(x, dtype, cuda), offset), dtype)
    assert_softmax_close(Y, ref, dtype, shape[-1], f"softmax_causal {dtype} {shape} off={offset}")
    # Masked entries are exactly +0.
    t1, t2 = shape[-2], shape[-1]
    i = np.arange(t1)[:, None]
    j = np.arange(t2)[None, :]
    masked = np.broadcast_to(j > i + offset, Y.shape)
    assert np.all(Y[masked] == 0)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,offset", [((1, 3, 4), 0), ((1, 2, 4), 2), ((2, 4, 33, 70), 5), ((6, 1, 9), 3),
                                          ((16, 16, 64, 203), 101), ((2, 3, 301, 4096), 3792),
                                          ((2, 3, 1024, 256), 0), ((2, 2, 8, 16), 15), ((1, 2, 4, 8), 100),
                                          ((50, 60, 3, 5), 0), ((50, 60, 3, 5), 1),
                                          # whole-vector rows (the lanes-over-masked-vectors kernel)
                                          ((3, 5, 33, 64), 0), ((2, 4, 70, 72), 5), ((1, 3, 1024, 1024), 0),
                                          ((70000, 1, 2, 64), 3)])
def test_causality_mask(oracle, xn, cuda, dtype, shape, offset):
    r = rng(len(shape) + offset)
    x = to_storage(randn(r, shape), dtype)
    ref = oracle.apply_causality_mask(x, offset, dtype)
    Y = xn.apply_causality_mask(to_device(x, dtype, cuda), offset)
    assert np.array_equal(from_device(Y, dtype), ref)


def test_softmax_decode_steps(oracle, xn, cuda):
    """Config 3: softmax over cached scores [16,16,1,t] bf16 for several t."""
    r = rng(11)
    for t in (1, 2, 31, 128, 256):
        x = to_storage(randn(r, (16, 16, 1, t), 1.0), "bf16")
        Y = xn.softmax(to_device(x, "bf16", cuda))
        assert_close(from_device(Y, "bf16"), oracle.softmax(x, "bf16"), "bf16", f"decode t={t}")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape,offset,scale", [((4, 8, 250, 250), 0, 0.125), ((16, 16, 1, 200), 199, 0.125),
                                                ((2, 3, 7, 7), None, 0.3), ((1, 2, 5, 20000), 19995, 0.125)])
def test_attn_softmax_scaled(oracle, xn, cuda, dtype, shape, offset, scale):
    """T(scores * scale), causal mask, softmax in one pass == the reference's
    `scale` (cpu_backend.rs:260-276), apply_causality_mask and softmax."""
    r = rng(sum(shape) + int(scale * 100))
    s = to_storage(randn(r, shape, 4.0), dtype)
    sc = to_storage(np.full(shape[-1], scale, dtype=np.float32), dtype)  # the T-typed scale
    scaled = oracle.broadcast_rows(s, sc, "mul", dtype)
    ref = oracle.softmax(scaled, dtype) if offset is None else oracle.softmax_causal(scaled, offset, dtype)
    scale_t = float(np.asarray(sc[:1]).view(np.float32)[0]) if dtype == "f32" else float(
        np.frombuffer(np.array([int(sc[0]) << 16], dtype=np.uint32).tobytes(), dtype=np.float32)[0])
    Y = xn.attn_softmax(to_device(s, dtype, cuda), scale_t, offset)
    assert_close(from_device(Y, dtype), ref, dtype, f"attn_softmax {dtype} {shape}")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("width", [8, 7, 6, 10])
def test_softmax_exp_every_input(oracle, xn, cuda, dtype, width):
    """Every non-positive 16-bit value v, through the vector path (rows of 8),
    the window path (rows of 10, starting at every offset within a 16-byte
    vector), the pair path (rows of 6) and the scalar path (rows of 7): rows
    [0, v, -inf, ...] have max 0, so
    e = T(exp(T(v - 0))) = T(exp(v)) and the row sum 1 + e is the same in any
    order. The outputs then equal the reference's bit for bit exactly when
    every T(exp(v)) does; the test reports how many of the 2^15 inputs differ."""
    bits = np.arange(0x8000, 0x10000, dtype=np.uint32).astype(np.uint16)  # sign set: -0 ... -NaN
    vals = bits.view(np.int16).astype(np.int32) & 0x7FFF
    exp_all_ones = 0x7F80 if dtype == "bf16" else 0x7C00
    keep = vals <= exp_all_ones  # drop NaN patterns; keep -inf
    v = bits[keep]
    n = v.size
    ninf = np.uint16(0xFF80 if dtype == "bf16" else 0xFC00)
    x = np.full((n, width), ninf, dtype=np.uint16)
    x[:, 0] = 0
    x[:, 1] = v
    ref = oracle.softmax(x, dtype)
    got = from_device(xn.softmax(to_device(x, dtype, cuda)), dtype)
    diff = np.nonzero(np.any(got != ref, axis=1))[0]
    print(f"{dtype}: {diff.size} of {n} inputs differ")
    assert diff.size == 0, f"first differing inputs: {[hex(int(b)) for b in v[diff[:8]]]}"
    if width in (8, 6, 10):
        # The same rows with the -inf columns masked by the fused causal mask
        # (one query row per slice, offset 1: columns >= 2 are not read)
        # instead of held in the data. A thread whose live values stay within
        # 86 of the row max then takes the flush-to-zero exp, so every input
        # v >= -86 goes through that form too.
        xm = x.copy()
        xm[:, 2:] = 0
        got_m = from_device(xn.softmax_causal(to_device(xm.reshape(n, 1, width), dtype, cuda), 1), dtype)
        diff = np.nonzero(np.any(got_m.reshape(n, width) != ref, axis=1))[0]
        print(f"{dtype} (causal): {diff.size} of {n} inputs differ")
        assert diff.size == 0, f"first differing inputs: {[hex(int(b)) for b in v[diff[:8]]]}"


@pytest.mark.parametrize("dtype,rows,cols", [("bf16", 6000, 4096), ("bf16", 13500, 2048), ("f16", 3000, 8192),
                                             ("bf16", 700, 32768), ("f32", 1100, 16384), ("f32", 5000, 1024),
                                             ("bf16", 30000, 250), ("f32", 30000, 250), ("f16", 4000, 1003),
                                             ("bf16", 3000, 2560), ("bf16", 3000, 3072), ("f16", 3000, 5120),
                                             ("bf16", 8000, 768), ("f16", 8000, 1536), ("f32", 8000, 1280),
                                             ("f32", 4000, 3072), ("f32", 3000, 5120)])
def test_softmax_many_rows_per_block(oracle, xn, cuda, dtype, rows, cols):
    """Enough rows that every block of the persistent kernels walks several:
    each shared-memory stage buffer of the staged kernel is refilled more than
    once (its barrier phases wrap). Also run in place (dst == src), which the
    ABI allows, and compared bit for bit with the out-of-place result."""
    r = rng(rows + cols)
    x = to_storage(randn(r, (rows, cols), 2.0), dtype)
    ref = oracle.softmax(x, dtype)
    X = to_device(x, dtype, cuda)
    Y = xn.softmax(X)
    assert_softmax_close(from_device(Y, dtype), ref, dtype, cols, f"softmax {dtype} {rows}x{cols}")
    xn.softmax_(X, X)
    assert np.array_equal(from_device(X, dtype), from_device(Y, dtype))


@pytest.mark.parametrize("dtype,shape,offset", [("bf16", (2, 2, 2048, 2048), 0), ("f16", (1, 3, 300, 4096), 7),
                                                ("f32", (1, 2, 1024, 9000), 0),
                                                # 5 / 6 vectors per thread, mostly masked and mostly live
                                                ("bf16", (1, 2, 2560, 2560), 0), ("bf16", (1, 2, 300, 5120), 4800),
                                                ("f16", (1, 2, 3072, 3072), 0), ("f16", (1, 2, 200, 3072), 2872)])
def test_softmax_causal_mostly_masked(oracle, xn, cuda, dtype, shape, offset):
    """Wide causal rows with fewer than 3/4 of their columns live on average
    (square prefill masks): the shared-memory-staged kernel then skips the
    arithmetic of masked vectors."""
    r = rng(sum(shape) + offset)
    x = to_storage(randn(r, shape, 2.0), dtype)
    ref = oracle.softmax_causal(x, offset, dtype)
    Y = from_device(xn.softmax_causal(to_device(x, dtype, cuda), offset), dtype)
    assert_close(Y, ref, dtype, f"softmax_causal {dtype} {shape} off={offset}")


@pytest.mark.parametrize("dtype,cols", [("bf16", 4096), ("f32", 4096), ("bf16", 1536), ("f16", 768),
                                        ("f32", 1280), ("f32", 5120)])
def test_softmax_causal_many_rows(oracle, xn, cuda, dtype, cols):
    """Causal rows of varying length (offset + i + 1 of `cols` columns, most of
    them ending inside a 16-byte vector), many per block; with and without the
    fused score scale."""
    shape, offset = (4, 8, 301, cols), cols - 301 - 3
    r = rng(77)
    x = to_storage(randn(r, shape, 2.0), dtype)
    ref = oracle.softmax_causal(x, offset, dtype)
    X = to_device(x, dtype, cuda)
    assert_close(from_device(xn.softmax_causal(X, offset), dtype), ref, dtype, f"softmax_causal {dtype} {shape}")
    sc = to_storage(np.full(shape[-1], 0.125, dtype=np.float32), dtype)
    ref_s = oracle.softmax_causal(oracle.broadcast_rows(x, sc, "mul", dtype), offset, dtype)
    assert_close(from_device(xn.attn_softmax(X, 0.125, offset), dtype), ref_s, dtype, f"attn_softmax {dtype} {shape}")
