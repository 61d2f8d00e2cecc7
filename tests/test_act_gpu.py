"""GPU parity: SiLU, GELU(erf) and the fused SwiGLU against the oracle
(cpu_backend.rs:184-258; SwiGLU = silu then mul, llama.rs:256-263)."""
import numpy as np
import pytest
import torch

from helpers import assert_close, from_device, gelu_erf_abs_bound, randn, rng, storage_to_f32, to_device, to_storage

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "bf16", "f16"]
SIZES = [1, 7, 1000, 4096 * 3 + 5, 1 << 20]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("op", ["silu", "gelu_erf"])
def test_unary(oracle, xn, cuda, dtype, n, op):
    r = rng(n + len(op))
    x = to_storage(randn(r, n, 3.0), dtype)
    ref = oracle.unary(x, op, dtype)
    Y = getattr(xn, op)(to_device(x, dtype, cuda))
    extra = gelu_erf_abs_bound(storage_to_f32(x, dtype)) if op == "gelu_erf" else None
    assert_close(from_device(Y, dtype), ref, dtype, f"{op} {dtype} n={n}", extra_abs=extra)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_unary_misaligned(oracle, xn, cuda, dtype):
    r = rng(3)
    n = 10001
    x = to_storage(randn(r, n, 2.0), dtype)
    X = to_device(np.concatenate([x[:1], x]), dtype, cuda)[1:]
    Y = torch.empty_like(X)
    xn.unary_(Y, X, "gelu_erf")
    assert_close(from_device(Y, dtype), oracle.unary(x, "gelu_erf", dtype), dtype, "gelu misaligned",
                 extra_abs=gelu_erf_abs_bound(storage_to_f32(x, dtype)))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (512, 5632), (64, 4096), (7, 1000)])
def test_swiglu_contiguous(oracle, xn, cuda, dtype, rows, cols):
    r = rng(rows * 3 + cols)
    g = to_storage(randn(r, (rows, cols), 2.0), dtype)
    u = to_storage(randn(r, (rows, cols)), dtype)
    ref = oracle.swiglu(g, u, dtype)
    Y = xn.swiglu(to_device(g, dtype, cuda), to_device(u, dtype, cuda))
    assert_close(from_device(Y, dtype), ref, dtype, f"swiglu {dtype} {rows}x{cols}")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,inter", [(64, 1024), (5, 24), (3, 7)])
def test_swiglu_packed_projection(oracle, xn, cuda, dtype, rows, inter):
    """gate and up as the two halves of one [rows, 2*I] projection output."""
    r = rng(rows + inter)
    gu = to_storage(randn(r, (rows, 2 * inter), 2.0), dtype)
    g, u = np.ascontiguousarray(gu[:, :inter]), np.ascontiguousarray(gu[:, inter:])
    ref = oracle.swiglu(g, u, dtype)
    GU = to_device(gu, dtype, cuda)
    Y = xn.swiglu(GU[:, :inter], GU[:, inter:])
    assert_close(from_device(Y, dtype), ref, dtype, "swiglu packed")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_swiglu_strided_past_the_grid_row_limit(oracle, xn, cuda, dtype):
    """A strided (packed-projection) SwiGLU over 70000 rows: the launch grid
    covers at most 65535 rows and the kernel loops over the rest."""
    rows, inter = 70000, 24
    r = rng(70000)
    gu = to_storage(randn(r, (rows, 2 * inter), 2.0), dtype)
    ref = oracle.swiglu(np.ascontiguousarray(gu[:, :inter]), np.ascontiguousarray(gu[:, inter:]), dtype)
    GU = to_device(gu, dtype, cuda)
    assert_close(from_device(xn.swiglu(GU[:, :inter], GU[:, inter:]), dtype), ref, dtype, "swiglu 70000 rows")


def test_config_shapes(oracle, xn, cuda):
    """Config 1 SwiGLU [1,512,5632] f32; config 2 GELU [4,250,2048] f32 and bf16;
    config 3 SiLU [16,4096] bf16."""
    r = rng(9)
    g, u = randn(r, (1, 512, 5632)), randn(r, (1, 512, 5632))
    Y = xn.swiglu(to_device(g, "f32", cuda), to_device(u, "f32", cuda))
    assert_close(from_device(Y, "f32"), oracle.swiglu(g, u, "f32"), "f32", "config1 swiglu")
    for dtype in ("f32", "bf16"):
        x = to_storage(randn(r, (4, 250, 2048)), dtype)
        Y = xn.gelu_erf(to_device(x, dtype, cuda))
        assert_close(from_device(Y, dtype), oracle.unary(x, "gelu_erf", dtype), dtype, f"config2 gelu {dtype}",
                     extra_abs=gelu_erf_abs_bound(storage_to_f32(x, dtype)))
    x = to_storage(randn(r, (16, 4096), 0.02), "bf16")
    Y = xn.silu(to_device(x, "bf16", cuda))
    assert_close(from_device(Y, "bf16"), oracle.unary(x, "silu", "bf16"), "bf16", "config3 silu")


@pytest.mark.parametrize("op", ["silu", "gelu_erf"])
def test_unary_bf16_exhaustive(oracle, xn, cuda, op):
    """Every finite bf16 input (the whole domain of the bf16 ops)."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    exp = (bits >> 7) & 0xFF
    x = bits[exp != 0xFF]  # drop inf / NaN
    ref = oracle.unary(x, op, "bf16")
    got = from_device(getattr(xn, op)(to_device(x, "bf16", cuda)), "bf16")
    extra = gelu_erf_abs_bound(storage_to_f32(x, "bf16")) if op == "gelu_erf" else None
    stats = assert_close(got, ref, "bf16", f"{op} bf16 exhaustive", extra_abs=extra)
    print(f"{op} bf16: {int(np.sum(got != ref))} of {x.size} inputs differ")
    # The only differences are from erff implementations (CUDA vs glibc).
    assert stats["exact_frac"] > 0.999, stats


def test_silu_f16_exhaustive(oracle, xn, cuda):
    """Every finite f16 input, bit for bit: the f16 SiLU takes exp(-s) from
    the hardware ex2 with a split of log2 e, and divides without the IEEE
    division routine (a reciprocal refined by the exact remainder), exact by
    the quotients' distance from f16 rounding midpoints."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    x = bits[((bits >> 10) & 0x1F) != 0x1F]
    ref = oracle.unary(x, "silu", "f16")
    got = from_device(xn.silu(to_device(x, "f16", cuda)), "f16")
    stats = assert_close(got, ref, "f16", "silu f16 exhaustive")
    print(f"silu f16: {int(np.sum(got != ref))} of {x.size} inputs differ")
    assert np.array_equal(got, ref), stats
    # Signed zeros and the quotients past exp's overflow (s <= -11.09: s / inf = -0).
    z = got[(x == 0x8000) | (x == 0x0000)]
    assert set(z.tolist()) == {0x8000, 0x0000}
    neg_big = storage_to_f32(x, "f16") < -11.5
    assert np.all(got[neg_big] == 0x8000)


def test_gelu_f16_exhaustive(oracle, xn, cuda):
    """Every finite f16 input through the 16-bit GELU(erf) (element pairs, the
    kernels' own erfc fit) against glibc's erff: within one ulp, or within the
    cancellation allowance |x| 2^-23 where x << 0."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    x = bits[((bits >> 10) & 0x1F) != 0x1F]
    ref = oracle.unary(x, "gelu_erf", "f16")
    got = from_device(xn.gelu_erf(to_device(x, "f16", cuda)), "f16")
    allow = gelu_erf_abs_bound(storage_to_f32(x, "f16"))
    stats = assert_close(got, ref, "f16", "gelu_erf f16 exhaustive", extra_abs=allow)
    print(f"gelu_erf f16: {int(np.sum(got != ref))} of {x.size} inputs differ")
    assert stats["exact_frac"] > 0.999, stats


def test_swiglu_f16_all_gates(oracle, xn, cuda):
    """Every finite f16 gate value against random up values."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    g = bits[((bits >> 10) & 0x1F) != 0x1F]
    u = to_storage(randn(rng(13), g.size, 2.0), "f16")
    ref = oracle.swiglu(g, u, "f16")
    got = from_device(xn.swiglu(to_device(g, "f16", cuda), to_device(u, "f16", cuda)), "f16")
    stats = assert_close(got, ref, "f16", "swiglu f16 all gates")
    print(f"swiglu f16: {int(np.sum(got != ref))} of {g.size} gates differ")
    assert np.array_equal(got, ref), stats


def test_swiglu_bf16_all_gates(oracle, xn, cuda):
    """Every finite bf16 gate value against random up values."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    g = bits[((bits >> 7) & 0xFF) != 0xFF]
    u = to_storage(randn(rng(12), g.size, 2.0), "bf16")
    ref = oracle.swiglu(g, u, "bf16")
    got = from_device(xn.swiglu(to_device(g, "bf16", cuda), to_device(u, "bf16", cuda)), "bf16")
    stats = assert_close(got, ref, "bf16", "swiglu bf16 all gates")
    print(f"swiglu bf16: {int(np.sum(got != ref))} of {g.size} gates differ")
    assert stats["exact_frac"] > 0.999, stats
