"""Tolerances and conversions shared by the parity tests.

Tolerances (per element, against the oracle's restatement of the reference
CPU backend):
  * gathers, RoPE, residual outputs: bit-exact (checked with array_equal);
  * f32: |gpu - ref| <= 1e-5 * max(|ref|, 1e-3 * rms(ref));
  * bf16 / f16: at most 1 ulp from the reference's result (bit distance), or,
    for results below 1e-3 * rms(ref), within one ulp of that floor.

The floor 1e-3 * rms(ref) only matters for outputs a thousand times smaller
than the tensor's typical value; above it the bound is the plain relative
one. Some ops get an extra absolute allowance, each derived from the
reference's own rounding error (see the functions below): LayerNorm, whose
x - mean and + bias cancel; GELU(erf), whose 1 + erf cancels; the decode
attention's weighted sum of V, whose terms cancel.

Every check is recorded in RECORDS (max relative error for f32, the ulp
histogram for 16-bit types); conftest prints a summary per op at the end of
the session.
"""
from __future__ import annotations

import numpy as np
import torch

NP_STORAGE = {"f32": np.float32, "bf16": np.uint16, "f16": np.uint16}
TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

F32_RTOL = 1e-5
F32_FLOOR = 1e-3  # fraction of rms(ref) below which errors are measured against that floor
HALF_MAX_ULP = 1
U32 = 2.0 ** -24  # unit roundoff of f32

# One entry per assert_close call: {"what", "dtype", "n", "max_rel" | "ulp_hist"}.
RECORDS: list[dict] = []


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


def sum_error_bound(n, abs_sum):
    """Rounding-error allowance of an f32 sum of n terms whose absolute values
    add up to abs_sum: 4 * sqrt(n) * 2^-24 * abs_sum.

    The reference adds row elements one after another (Iterator::sum,
    cpu_backend.rs:702,727-738; the matmul's k loop), the kernels in a fixed
    tree or in interleaved partial sums. Each order's error is a sum of n
    roundings of at most 2^-24 of a partial sum; with independent rounding
    signs it is about sqrt(n) * 2^-24 * abs_sum / 3 (partial sums growing
    linearly), so 4 * sqrt(n) * 2^-24 covers both orders' errors with a wide
    margin, while staying 1/sqrt(n)-th of the worst-case n * 2^-24 bound."""
    return 4.0 * np.sqrt(np.asarray(n, dtype=np.float64)) * U32 * abs_sum


def layer_norm_abs_bound(h_f32: np.ndarray, w_f32: np.ndarray | None, eps: float,
                         remove_mean: bool = True) -> np.ndarray:
    """Absolute allowance for LayerNorm outputs (per element, shape of h).

    LayerNorm computes y = (h - mean) * inv * w + b with mean and var from f32
    row sums (cpu_backend.rs:711-750). The reference's sums are sequential,
    the kernels' are trees, so mean differs by up to sum_error_bound(n,
    sum|h|) / n and inv by the same relative amount as var. (h - mean) cancels
    for h near the mean and + b cancels for (h - mean) * inv * w near -b, so
    those differences are absolute errors of the output:
      |dmean| * inv * |w|   +   |(h - mean) * inv * w| * (relative error of inv).
    Everything else in the formula is the same f32 operation on both sides."""
    h = h_f32.astype(np.float64)
    n = h.shape[-1]
    w = np.ones(n) if w_f32 is None else w_f32.astype(np.float64)
    mean = h.mean(axis=-1, keepdims=True)
    var = ((h - mean) ** 2).mean(axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(var + eps)
    dmean = sum_error_bound(n, np.abs(h).sum(axis=-1, keepdims=True)) / n
    c = (h - mean) if remove_mean else h
    rel_inv = sum_error_bound(n, 1.0)  # var's sum has non-negative terms: relative error
    return dmean * inv * np.abs(w) * (1.0 if remove_mean else 0.0) + np.abs(c * inv * w) * rel_inv


def attention_abs_bound(probs_f32: np.ndarray, v_f32: np.ndarray) -> np.ndarray:
    """Absolute allowance for out = sum_j p_j v_j (decode attention): the
    reference's matmul adds the products in key order, the kernel in
    interleaved partial sums; the terms cancel, so the difference is bounded
    by sum_error_bound(kv, sum_j |p_j v_j|). probs [b, h, t, kv], v [b, h, kv, d]
    -> [b, t, h, d]."""
    p = np.abs(probs_f32.astype(np.float64))
    a = np.abs(v_f32.astype(np.float64))
    kv = p.shape[-1]
    s = np.matmul(p, a)  # [b, h, t, d]
    return np.transpose(sum_error_bound(kv, s), (0, 2, 1, 3))


def _record(rec: dict) -> dict:
    RECORDS.append(rec)
    return rec


def assert_close(got: np.ndarray, ref: np.ndarray, dtype: str, what: str = "",
                 extra_abs: np.ndarray | None = None) -> dict:
    """Asserts the tolerance for dtype; returns (and records) a summary of the
    differences.

    extra_abs (optional, per element): an absolute error the op's own
    definition leaves open (gelu_erf_abs_bound, layer_norm_abs_bound,
    attention_abs_bound), added to the tolerance."""
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    extra = None if extra_abs is None else np.broadcast_to(extra_abs, ref.shape)
    if dtype == "f32":
        g, r = got.astype(np.float64), ref.astype(np.float64)
        finite = np.isfinite(r)
        assert np.array_equal(np.isfinite(g), finite), f"{what}: non-finite pattern differs"
        assert np.array_equal(g[~finite], r[~finite], equal_nan=True), f"{what}: non-finite values differ"
        if not finite.any():
            return _record({"what": what, "dtype": dtype, "n": int(ref.size), "max_rel": 0.0})
        rms = float(np.sqrt(np.mean(r[finite] ** 2)))
        denom = np.maximum(np.abs(r), F32_FLOOR * rms)
        denom = np.where(denom == 0, 1.0, denom)
        err = np.abs(g - r)
        raw = np.where(finite, err / denom, 0.0)
        if extra is not None:
            err = np.maximum(err - extra, 0.0)
        rel = np.where(finite, err / denom, 0.0)
        mx = float(rel.max())
        assert mx <= F32_RTOL, (f"{what}: max relative error {mx:.3e} > {F32_RTOL} at "
                                f"{np.unravel_index(rel.argmax(), rel.shape)}")
        return _record({"what": what, "dtype": dtype, "n": int(ref.size), "max_rel": mx,
                        "max_rel_raw": float(raw.max()), "exact_frac": float(np.mean(got == ref))})
    d = ulp_distance(got, ref)
    bad = d > HALF_MAX_ULP
    n_allowed = 0
    if bad.any():
        g = storage_to_f32(got, dtype).astype(np.float64)
        r = storage_to_f32(ref, dtype).astype(np.float64)
        fin = np.isfinite(r)
        rms = float(np.sqrt(np.mean(r[fin] ** 2))) if fin.any() else 0.0
        # One ulp at max(|ref|, 1e-3 * rms), plus the formula's own uncertainty if given.
        tol = half_ulp(np.maximum(np.abs(r), F32_FLOOR * rms), dtype)
        if extra is not None:
            tol = tol + extra
        ok = np.abs(g - r) <= tol
        n_allowed = int((bad & ok).sum())
        bad &= ~ok
    mx = int(d.max()) if d.size else 0
    assert not bad.any(), f"{what}: max ulp distance {mx} > {HALF_MAX_ULP} (count {int(bad.sum())})"
    hist = {"0": int((d == 0).sum()), "1": int((d == 1).sum()), ">1 (within allowance)": n_allowed}
    return _record({"what": what, "dtype": dtype, "n": int(ref.size), "max_ulp": mx, "ulp_hist": hist,
                    "exact_frac": float(np.mean(d == 0)) if d.size else 1.0})


def randn(r: np.random.Generator, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    return (r.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(np.float32)
