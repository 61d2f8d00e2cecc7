"""Tolerances and conversions shared by the parity tests.

Tolerances:
  * gathers: bit-exact;
  * f32: |gpu - ref| <= 1e-5 * max(|ref|, rms(ref)): relative error, measured
    against the output tensor's RMS for elements below it;
  * bf16 / f16: at most 1 ulp from the reference CPU backend's own result,
    the ulp taken at max(|ref|, rms(ref)).

Why the RMS floor: the reference accumulates row sums sequentially in f32
(cpu_backend.rs:702,727-738), the kernels in a fixed tree. Both carry an error
of about sqrt(n) * 2^-24 of the row scale, and outputs that are differences of
row-scale values (LayerNorm's x - mean, near-zero results) inherit it as an
absolute error, so their element-wise relative error is unbounded while the
error relative to the output's scale stays ~1e-6.
"""
from __future__ import annotations

import numpy as np
import torch

NP_STORAGE = {"f32": np.float32, "bf16": np.uint16, "f16": np.uint16}
TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

F32_RTOL = 1e-5
F32_FLOOR = 1.0  # fraction of rms(ref) below which errors are measured against rms(ref)
HALF_MAX_ULP = 1


def half_ulp(v: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of bf16 / f16 values at magnitude v (v > 0)."""
    bits = 7 if dtype == "bf16" else 10
    e = np.floor(np.log2(np.maximum(v, 1e-38)))
    return np.exp2(e - bits)


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def to_storage(a_f32: np.ndarray, dtype: str) -> np.ndarray:
    """f32 values rounded (RNE) to dtype, as numpy storage (uint16 bits for halves)."""
    t = torch.from_numpy(np.ascontiguousarray(a_f32, dtype=np.float32)).to(TORCH_DTYPE[dtype])
    if dtype == "f32":
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def storage_to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return a.astype(np.float32)
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(TORCH_DTYPE[dtype])
    return t.float().numpy()


def to_device(a: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype != "f32":
        t = t.view(torch.int16).view(TORCH_DTYPE[dtype])
    return t.to(device)


def from_device(t: torch.Tensor, dtype: str) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if dtype == "f32":
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units of the last place between 16-bit float bit patterns."""
    def key(x):
        v = x.astype(np.int32)
        mag = v & 0x7FFF
        return np.where(v & 0x8000, -mag, mag)
    return np.abs(key(a) - key(b))


def gelu_erf_abs_bound(x_f32: np.ndarray) -> np.ndarray:
    """Absolute uncertainty of the reference GELU formula x*0.5*(1+erf(x/sqrt2)).

    For x << 0, 1 + erf(x/sqrt2) cancels: erf is near -1, where one f32 ulp is
    2^-24, and erff implementations (the reference's `libm` crate, glibc, CUDA)
    agree only to a few ulps. The formula's result is therefore defined only
    to 0.5*|x| * 4 ulps = |x| * 2^-23 in absolute terms; the GELU tests add
    this to the f32 / 1-ulp tolerance.
    """
    return np.abs(x_f32.astype(np.float64)) * 2.0 ** -23


def assert_close(got: np.ndarray, ref: np.ndarray, dtype: str, what: str = "",
                 extra_abs: np.ndarray | None = None) -> dict:
    """Asserts the tolerance for dtype; returns a summary of the differences.

    extra_abs (optional, per element): an absolute error the op's own
    definition leaves open (see gelu_erf_abs_bound), added to the tolerance."""
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    extra = None if extra_abs is None else np.broadcast_to(extra_abs, ref.shape)
    if dtype == "f32":
        g, r = got.astype(np.float64), ref.astype(np.float64)
        finite = np.isfinite(r)
        assert np.array_equal(np.isfinite(g), finite), f"{what}: non-finite pattern differs"
        if not finite.any():
            return {"max_rel": 0.0}
        rms = float(np.sqrt(np.mean(r[finite] ** 2))) if finite.any() else 0.0
        denom = np.maximum(np.abs(r), F32_FLOOR * rms)
        denom = np.where(denom == 0, 1.0, denom)
        err = np.abs(g - r)
        if extra is not None:
            err = np.maximum(err - extra, 0.0)
        rel = np.where(finite, err / denom, 0.0)
        mx = float(rel.max())
        assert mx <= F32_RTOL, f"{what}: max relative error {mx:.3e} > {F32_RTOL} at {np.unravel_index(rel.argmax(), rel.shape)}"
        return {"max_rel": mx, "exact_frac": float(np.mean(got == ref))}
    d = ulp_distance(got, ref)
    bad = d > HALF_MAX_ULP
    if bad.any():
        g = storage_to_f32(got, dtype).astype(np.float64)
        r = storage_to_f32(ref, dtype).astype(np.float64)
        fin = np.isfinite(r)
        rms = float(np.sqrt(np.mean(r[fin] ** 2))) if fin.any() else 0.0
        # One ulp at max(|ref|, rms), plus the formula's own uncertainty if given.
        tol = half_ulp(np.maximum(np.abs(r), F32_FLOOR * rms), dtype)
        if extra is not None:
            tol = tol + extra
        bad &= ~(np.abs(g - r) <= tol)
    mx = int(d.max()) if d.size else 0
    assert not bad.any(), f"{what}: max ulp distance {mx} > {HALF_MAX_ULP} (count {int(bad.sum())})"
    return {"max_ulp": mx, "exact_frac": float(np.mean(d == 0)) if d.size else 1.0}


def randn(r: np.random.Generator, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    return (r.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(np.float32)
