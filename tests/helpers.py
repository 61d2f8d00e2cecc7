"""Tolerances and conversions shared by the parity tests.

Tolerances:
  * gathers: bit-exact;
  * f32: |gpu - ref| <= 1e-5 * max(|ref|, 1e-3 * rms(ref))  (relative error with
    a floor for near-zero outputs);
  * bf16 / f16: at most 1 ulp from the reference CPU backend's own result.
"""
from __future__ import annotations

import numpy as np
import torch

NP_STORAGE = {"f32": np.float32, "bf16": np.uint16, "f16": np.uint16}
TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

F32_RTOL = 1e-5
F32_FLOOR = 1e-3
HALF_MAX_ULP = 1


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


def assert_close(got: np.ndarray, ref: np.ndarray, dtype: str, what: str = "") -> dict:
    """Asserts the tolerance for dtype; returns a summary of the differences."""
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    if dtype == "f32":
        g, r = got.astype(np.float64), ref.astype(np.float64)
        finite = np.isfinite(r)
        assert np.array_equal(np.isfinite(g), finite), f"{what}: non-finite pattern differs"
        if not finite.any():
            return {"max_rel": 0.0}
        rms = float(np.sqrt(np.mean(r[finite] ** 2))) if finite.any() else 0.0
        denom = np.maximum(np.abs(r), F32_FLOOR * rms)
        denom = np.where(denom == 0, 1.0, denom)
        rel = np.where(finite, np.abs(g - r) / denom, 0.0)
        mx = float(rel.max())
        assert mx <= F32_RTOL, f"{what}: max relative error {mx:.3e} > {F32_RTOL} at {np.unravel_index(rel.argmax(), rel.shape)}"
        return {"max_rel": mx, "exact_frac": float(np.mean(got == ref))}
    d = ulp_distance(got, ref)
    mx = int(d.max()) if d.size else 0
    assert mx <= HALF_MAX_ULP, f"{what}: max ulp distance {mx} > {HALF_MAX_ULP} (count {int((d > HALF_MAX_ULP).sum())})"
    return {"max_ulp": mx, "exact_frac": float(np.mean(d == 0)) if d.size else 1.0}


def randn(r: np.random.Generator, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    return (r.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(np.float32)
