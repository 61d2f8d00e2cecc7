"""Runs the reference's known-answer cases (tests/golden/known_answers.json)
against either the CPU oracle or the GPU kernels, in f32 as the reference
tests do."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "known_answers.json"


def load_cases():
    return json.loads(GOLDEN.read_text())["cases"]


def _arr(v, shape=None):
    a = np.array([float(x) for x in np.ravel(np.array(v, dtype=object))], dtype=np.float32)
    return a.reshape(shape) if shape is not None else a


def _expected(case):
    vals = [(-np.inf if x == "-inf" else float(x)) for x in np.ravel(np.array(case["expected"], dtype=object))]
    return np.array(vals, dtype=np.float32)


class OracleRunner:
    def __init__(self, oracle):
        self.o = oracle

    def softmax(self, x):
        return self.o.softmax(x, "f32")

    def rms_norm(self, x, alpha, eps):
        return self.o.rms_norm(x, alpha, eps, "f32")

    def layer_norm(self, x, w, b, eps):
        return self.o.layer_norm(x, w, b, eps, "f32")

    def silu(self, x):
        return self.o.unary(x, "silu", "f32")

    def index_select(self, x, ids, dim):
        return self.o.index_select(x, ids, dim)

    def causality_mask(self, x, offset):
        return self.o.apply_causality_mask(x, offset, "f32")

    def rope(self, x, cos, sin, pos):
        return self.o.rope(x, cos, sin, pos, "f32")


class GpuRunner:
    def __init__(self, xn, device):
        import torch

        self.xn, self.dev, self.torch = xn, device, torch

    def _t(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a)).to(self.dev)

    def _n(self, t):
        return t.cpu().numpy()

    def softmax(self, x):
        return self._n(self.xn.softmax(self._t(x)))

    def rms_norm(self, x, alpha, eps):
        return self._n(self.xn.rms_norm(self._t(x), self._t(alpha), eps))

    def layer_norm(self, x, w, b, eps):
        return self._n(self.xn.layer_norm(self._t(x), self._t(w), self._t(b), eps))

    def silu(self, x):
        return self._n(self.xn.silu(self._t(x)))

    def index_select(self, x, ids, dim):
        return self._n(self.xn.index_select(self._t(x), list(ids), dim))

    def causality_mask(self, x, offset):
        return self._n(self.xn.apply_causality_mask(self._t(x), offset))

    def rope(self, x, cos, sin, pos):
        return self._n(self.xn.rope(self._t(x), self._t(cos), self._t(sin), pos))


def run_case(case, runner):
    """Evaluates one case; raises AssertionError on a mismatch."""
    op = case["op"]
    exp = _expected(case)
    if op == "softmax":
        x = _arr(case["x"]).reshape(len(case["x"]), -1)
        got = runner.softmax(x)
        assert np.allclose(got.ravel(), exp, atol=case["tol"], rtol=0), (case["name"], got, exp)
        if "row_sum_tol" in case:
            assert np.all(np.abs(got.sum(-1) - 1.0) < case["row_sum_tol"])
    elif op in ("rms_norm", "layer_norm"):
        x = _arr(case["x"]).reshape(len(case["x"]), -1)
        if op == "rms_norm":
            got = runner.rms_norm(x, _arr(case["alpha"]), case["eps"])
        else:
            got = runner.layer_norm(x, _arr(case["weight"]), _arr(case["bias"]), case["eps"])
        assert np.allclose(got.ravel(), exp, atol=case["tol"], rtol=0), (case["name"], got, exp)
    elif op == "silu":
        got = runner.silu(_arr(case["x"]))
        assert np.allclose(got.ravel(), exp, atol=case["tol"], rtol=0), (case["name"], got, exp)
    elif op == "index_select":
        x = _arr(case["x"], case["shape"])
        got = runner.index_select(x, case["ids"], case["dim"])
        assert list(got.shape) == case["expected_shape"], (case["name"], got.shape)
        assert np.array_equal(got.ravel(), exp), (case["name"], got, exp)
    elif op == "causality_mask":
        x = np.full(case["shape"], case["fill"], dtype=np.float32)
        got = runner.causality_mask(x, case["offset"])
        assert np.array_equal(got.ravel(), exp), (case["name"], got, exp)
    elif op == "rope":
        x = _arr(case["x"], case["shape"])
        cos = _arr(case["cos"], case["table_shape"])
        sin = _arr(case["sin"], case["table_shape"])
        got = runner.rope(x, cos, sin, case["pos"])
        assert np.allclose(got.ravel(), exp, atol=case["tol"], rtol=0), (case["name"], got, exp)
        if case.get("not_identity"):
            assert not np.allclose(got.ravel(), x.ravel(), atol=1e-5)
    else:
        raise ValueError(f"unknown op {op}")
