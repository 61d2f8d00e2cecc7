"""GPU parity: RMSNorm / LayerNorm (with the fused residual and layer-scale
prologue) against the oracle's restatement of the reference composite
(broadcast_mul -> add -> norm, mimi.rs:1433-1439 / llama.rs:310-313)."""
import numpy as np
import pytest
import torch

from helpers import (assert_close, from_device, layer_norm_abs_bound, randn, rng, storage_to_f32, to_device,
                     to_storage)

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "bf16", "f16"]
# Register path (vector and scalar), tiny rows, ragged widths, and the multi-pass
# path for rows wider than 32768 elements.
# (512, 768) / (512, 1536): several rows per block with 3 and 6 accesses per
# thread; (8, 10240): the 512-thread shape with 6 accesses (f32).
SHAPES = [(1, 3), (2, 3), (7, 64), (129, 100), (33, 1000), (16, 1024), (512, 2048), (5, 4096),
          (3, 5000), (4, 16384), (2, 40000), (512, 768), (512, 1536), (8, 10240), (300, 250)]


def ln_allowance(h, w, dtype, remove_mean=True, eps=1e-5):
    """LayerNorm's derived absolute allowance (helpers.layer_norm_abs_bound) for
    the normalised input h (storage) and weight w (storage)."""
    return layer_norm_abs_bound(storage_to_f32(h, dtype), storage_to_f32(w, dtype), eps, remove_mean)


def _inputs(seed, rows, cols, dtype, ln=False):
    r = rng(seed)
    x = to_storage(randn(r, (rows, cols), 1.0, 0.5 if ln else 0.0), dtype)
    br = to_storage(randn(r, (rows, cols)), dtype)
    w = to_storage(randn(r, cols, 0.02, 1.0), dtype)
    b = to_storage(randn(r, cols, 0.1), dtype)
    ls = to_storage(r.uniform(0, 0.1, cols).astype(np.float32), dtype)
    return x, br, w, b, ls


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("variant", ["plain", "residual", "residual_ls"])
def test_rms_norm(oracle, xn, cuda, dtype, rows, cols, variant):
    x, br, w, _, ls = _inputs(rows * 7 + cols, rows, cols, dtype)
    eps = 1e-5
    branch = None if variant == "plain" else br
    lsc = ls if variant == "residual_ls" else None
    ref_y, ref_h = oracle.rms_norm_residual(x, branch, w, eps, dtype, layer_scale=lsc)
    X, W = to_device(x, dtype, cuda), to_device(w, dtype, cuda)
    if branch is None:
        Y = xn.rms_norm(X, W, eps)
    else:
        Y, H = xn.rms_norm_residual(X, to_device(br, dtype, cuda), W, eps,
                                    layer_scale=None if lsc is None else to_device(lsc, dtype, cuda))
        assert np.array_equal(from_device(H, dtype), ref_h), "residual output must be bit-exact"
    assert_close(from_device(Y, dtype), ref_y, dtype, f"rms_norm {dtype} {rows}x{cols} {variant}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("variant", ["plain", "residual", "residual_ls", "no_mean"])
def test_layer_norm(oracle, xn, cuda, dtype, rows, cols, variant):
    x, br, w, b, ls = _inputs(rows * 11 + cols, rows, cols, dtype, ln=True)
    eps = 1e-5
    branch = br if variant.startswith("residual") else None
    lsc = ls if variant == "residual_ls" else None
    rm = variant != "no_mean"
    ref_y, ref_h = oracle.layer_norm_residual(x, branch, w, b, eps, dtype, layer_scale=lsc, remove_mean=rm)
    X, W, B = (to_device(a, dtype, cuda) for a in (x, w, b))
    if branch is None:
        Y = xn.layer_norm_rm(X, W, B, eps, rm)
    else:
        Y, H = xn.layer_norm_residual(X, to_device(br, dtype, cuda), W, B, eps,
                                      layer_scale=None if lsc is None else to_device(lsc, dtype, cuda),
                                      remove_mean=rm)
        assert np.array_equal(from_device(H, dtype), ref_h), "residual output must be bit-exact"
    h = x if branch is None else ref_h
    assert_close(from_device(Y, dtype), ref_y, dtype, f"layer_norm {dtype} {rows}x{cols} {variant}",
                 extra_abs=ln_allowance(h, w, dtype, rm))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_norm_misaligned_and_inplace(oracle, xn, cuda, dtype):
    """Unaligned views take the scalar path; residual_out may alias src."""
    rows, cols = 37, 4096
    x, br, w, b, ls = _inputs(5, rows, cols, dtype)
    ref_y, ref_h = oracle.rms_norm_residual(x, br, w, 1e-5, dtype, layer_scale=ls)
    big = torch.empty(rows * cols + 1, dtype=to_device(x, dtype, cuda).dtype, device=cuda)
    X = big[1:].view(rows, cols)
    X.copy_(to_device(x, dtype, cuda))
    Y = torch.empty_like(X)
    xn.rms_norm_(Y, X, to_device(w, dtype, cuda), 1e-5, branch=to_device(br, dtype, cuda),
                 layer_scale=to_device(ls, dtype, cuda), residual_out=X)
    assert np.array_equal(from_device(X, dtype), ref_h)
    assert_close(from_device(Y, dtype), ref_y, dtype, "rms_norm misaligned in-place")
    # LayerNorm in place on an aligned buffer (dst == src).
    ref_ln = oracle.layer_norm(x, w, b, 1e-5, dtype)
    X2 = to_device(x, dtype, cuda)
    xn.layer_norm_(X2, X2, to_device(w, dtype, cuda), to_device(b, dtype, cuda), 1e-5)
    assert_close(from_device(X2, dtype), ref_ln, dtype, "layer_norm in place", extra_abs=ln_allowance(x, w, dtype))


def test_norm_config_shapes(oracle, xn, cuda):
    """Benchmark config 1 (f32 RMSNorm [1,512,2048]) and config 2 (LN + layer-scale
    + residual on [4,250,512], f32 and bf16)."""
    r = rng(100)
    x = randn(r, (1, 512, 2048))
    w = randn(r, 2048, 0.02, 1.0)
    Y = xn.rms_norm(to_device(x, "f32", cuda), to_device(w, "f32", cuda), 1e-5)
    assert_close(from_device(Y, "f32"), oracle.rms_norm(x, w, 1e-5, "f32"), "f32", "config1 rms_norm")
    for dtype in ("f32", "bf16"):
        x = to_storage(randn(r, (4, 250, 512)), dtype)
        br = to_storage(randn(r, (4, 250, 512)), dtype)
        w = to_storage(randn(r, 512, 0.02, 1.0), dtype)
        b = to_storage(randn(r, 512, 0.02), dtype)
        ls = to_storage(r.uniform(0, 0.1, 512).astype(np.float32), dtype)
        ref_y, ref_h = oracle.layer_norm_residual(x, br, w, b, 1e-5, dtype, layer_scale=ls)
        Y, H = xn.layer_norm_residual(*(to_device(a, dtype, cuda) for a in (x, br, w, b)), 1e-5,
                                      layer_scale=to_device(ls, dtype, cuda))
        assert np.array_equal(from_device(H, dtype), ref_h)
        assert_close(from_device(Y, dtype), ref_y, dtype, f"config2 layer_norm {dtype}",
                     extra_abs=ln_allowance(ref_h, w, dtype))


def test_norm_deterministic(xn, cuda):
    r = rng(101)
    X = to_device(to_storage(randn(r, (1000, 4096)), "bf16"), "bf16", cuda)
    W = to_device(to_storage(randn(r, 4096, 0.02, 1.0), "bf16"), "bf16", cuda)
    a = xn.rms_norm(X, W, 1e-5)
    b = xn.rms_norm(X, W, 1e-5)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(1000, 512), (7, 100), (3, 1), (70000, 24), (2048, 256), (513, 64),
                                       (4, 4104)])
@pytest.mark.parametrize("with_ls", [True, False])
def test_residual_add(oracle, xn, cuda, dtype, rows, cols, with_ls):
    """x + LayerScale(branch), bit-exact (mimi.rs:1441-1444)."""
    x, br, _, _, ls = _inputs(rows + cols, rows, cols, dtype)
    ref = oracle.residual_prologue(x, br, ls if with_ls else None, dtype)
    Y = xn.residual_add(to_device(x, dtype, cuda), to_device(br, dtype, cuda),
                        to_device(ls, dtype, cuda) if with_ls else None)
    assert np.array_equal(from_device(Y, dtype), ref)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(1000, 250), (64, 1002), (6, 2046), (33, 10), (257, 36), (4, 4094),
                                       (512, 100), (1024, 170), (256, 126), (8, 250), (1002, 250)])
@pytest.mark.parametrize("variant", ["rms", "rms_residual", "rms_residual_ls", "ln", "ln_residual_ls", "ln_no_mean"])
def test_norm_narrow_accesses(oracle, xn, cuda, dtype, rows, cols, variant):
    """Rows whose byte width is a multiple of 8 or 4 but not 16 (16-bit rows of
    even width such as Mimi's 250 scores, f32 rows of even width). RMSNorm
    rows whose count divides into runs of 4 rows (f32: 2 or 4) that start on
    16-byte boundaries (1000 x 250, 1024 x 170, 256 x 126, 8 x 250; f32 also
    512 x 100) take the run kernel's 16-byte accesses, some holding the end of
    one row and the start of the next; the rest (LayerNorm, 1002 x 250, ...)
    take 8- and 4-byte accesses with the vector kernel's arithmetic."""
    x, br, w, b, ls = _inputs(rows * 5 + cols, rows, cols, dtype, ln=variant.startswith("ln"))
    eps = 1e-5
    branch = br if "residual" in variant else None
    lsc = ls if "residual_ls" in variant else None
    X, W, B = (to_device(a, dtype, cuda) for a in (x, w, b))
    BR = None if branch is None else to_device(br, dtype, cuda)
    LS = None if lsc is None else to_device(lsc, dtype, cuda)
    if variant.startswith("rms"):
        ref_y, ref_h = oracle.rms_norm_residual(x, branch, w, eps, dtype, layer_scale=lsc)
        Y = torch.empty_like(X)
        H = torch.empty_like(X) if branch is not None else None
        xn.rms_norm_(Y, X, W, eps, branch=BR, layer_scale=LS, residual_out=H)
        allow = None
    else:
        rm = variant != "ln_no_mean"
        ref_y, ref_h = oracle.layer_norm_residual(x, branch, w, b, eps, dtype, layer_scale=lsc, remove_mean=rm)
        if branch is None:
            Y = xn.layer_norm_rm(X, W, B, eps, rm)
            H = None
        else:
            Y, H = xn.layer_norm_residual(X, BR, W, B, eps, layer_scale=LS, remove_mean=rm)
        allow = ln_allowance(ref_h if branch is not None else x, w, dtype, rm)
    if H is not None:
        assert np.array_equal(from_device(H, dtype), ref_h), "residual output must be bit-exact"
    assert_close(from_device(Y, dtype), ref_y, dtype, f"{variant} {dtype} {rows}x{cols} narrow", extra_abs=allow)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_norm_view_4_byte_aligned(oracle, xn, cuda, dtype):
    """A [rows, 4096] view starting 4 bytes past a 16-byte boundary: 4-byte
    (16-bit) / scalar (f32) accesses; results as the aligned tensor's."""
    rows, cols = 37, 4096
    x, br, w, b, ls = _inputs(9, rows, cols, dtype)
    ref_y = oracle.rms_norm(x, w, 1e-5, dtype)
    t = to_device(x, dtype, cuda)
    step = 4 // t.element_size()
    big = torch.empty(rows * cols + step, dtype=t.dtype, device=cuda)
    X = big[step:].view(rows, cols)
    X.copy_(t)
    Y = torch.empty_like(X)
    xn.rms_norm_(Y, X, to_device(w, dtype, cuda), 1e-5)
    assert_close(from_device(Y, dtype), ref_y, dtype, f"rms_norm {dtype} 4-byte-aligned view")
    ref_ln = oracle.layer_norm(x, w, b, 1e-5, dtype)
    Z = torch.empty_like(X)
    xn.layer_norm_(Z, X, to_device(w, dtype, cuda), to_device(b, dtype, cuda), 1e-5)
    assert_close(from_device(Z, dtype), ref_ln, dtype, f"layer_norm {dtype} 4-byte-aligned view",
                 extra_abs=ln_allowance(x, w, dtype))
