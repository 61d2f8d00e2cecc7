"""Writes tests/golden/known_answers.json: the reference's own known-answer
tests for the fused-op path, as data.

Each case restates one assertion of mimi-rs/tests/cuda_tests.rs or
mimi-rs/tests/tensor_tests.rs (cited per case): its input, its expected output
(evaluated here in f32 exactly as the test's expression does) and its
tolerance. The oracle must reproduce every case (tests/test_oracle.py), and so
must the GPU kernels (tests/test_known_answers_gpu.py).

Run: python tests/golden/make_known_answers.py
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

f32 = np.float32
OUT = Path(__file__).resolve().with_name("known_answers.json")


def rms_expected(row, alpha, eps=1e-5):
    # cuda_tests.rs:371-375: scale = 1 / (sum(x^2)/n + eps).sqrt(); expect x * scale * alpha
    ms = f32(sum(f32(v) * f32(v) for v in row)) / f32(len(row))
    scale = f32(1.0) / np.sqrt(f32(ms + f32(eps)))
    return [float(f32(v) * scale * f32(a)) for v, a in zip(row, alpha)]


def ln_expected(row, w, b, eps=1e-5):
    # cuda_tests.rs:417-423: mean, biased var, inv_std = 1 / (var + eps).sqrt()
    n = f32(len(row))
    mean = f32(sum(f32(v) for v in row)) / n
    var = f32(sum((f32(v) - mean) ** 2 for v in row)) / n
    inv = f32(1.0) / np.sqrt(f32(var + f32(eps)))
    return [float((f32(v) - mean) * inv * f32(wi) + f32(bi)) for v, wi, bi in zip(row, w, b)]


NEG_INF = "-inf"


def cases():
    c = []
    c.append(dict(name="softmax_2x3", source="mimi-rs/tests/cuda_tests.rs:323-342", op="softmax",
                  x=[[1, 2, 3], [1, 2, 3]],
                  expected=[[0.0900306, 0.2447285, 0.6652409]] * 2, tol=1e-4, row_sum_tol=1e-5))
    c.append(dict(name="softmax_single_row", source="mimi-rs/tests/cuda_tests.rs:344-355", op="softmax",
                  x=[[0, 0, 0]], expected=[[1 / 3, 1 / 3, 1 / 3]], tol=1e-5))
    c.append(dict(name="rms_norm", source="mimi-rs/tests/cuda_tests.rs:361-384", op="rms_norm",
                  x=[[1, 2, 3], [4, 5, 6]], alpha=[1, 1, 1], eps=1e-5,
                  expected=[rms_expected([1, 2, 3], [1, 1, 1]), rms_expected([4, 5, 6], [1, 1, 1])], tol=1e-4))
    c.append(dict(name="rms_norm_with_scale", source="mimi-rs/tests/cuda_tests.rs:386-401", op="rms_norm",
                  x=[[1, 2, 3]], alpha=[2, 2, 2], eps=1e-5,
                  expected=[rms_expected([1, 2, 3], [2, 2, 2])], tol=1e-4))
    c.append(dict(name="layer_norm", source="mimi-rs/tests/cuda_tests.rs:407-433", op="layer_norm",
                  x=[[1, 2, 3], [4, 5, 6]], weight=[1, 1, 1], bias=[0, 0, 0], eps=1e-5,
                  expected=[ln_expected([1, 2, 3], [1] * 3, [0] * 3), ln_expected([4, 5, 6], [1] * 3, [0] * 3)],
                  tol=1e-4))
    c.append(dict(name="layer_norm_with_affine", source="mimi-rs/tests/cuda_tests.rs:435-452", op="layer_norm",
                  x=[[1, 2, 3]], weight=[2, 2, 2], bias=[1, 1, 1], eps=1e-5,
                  expected=[ln_expected([1, 2, 3], [2] * 3, [1] * 3)], tol=1e-4))
    c.append(dict(name="silu", source="mimi-rs/tests/cuda_tests.rs:146-156", op="silu",
                  x=[0.0, 1.0, -1.0], expected=[0.0, 0.7310586, -0.26894143], tol=1e-5))
    c.append(dict(name="index_select_1d", source="mimi-rs/tests/cuda_tests.rs:598-609", op="index_select",
                  x=[10, 20, 30, 40, 50], shape=[5], ids=[0, 2, 4], dim=0, expected=[10, 30, 50],
                  expected_shape=[3]))
    c.append(dict(name="index_select_2d_dim0", source="mimi-rs/tests/cuda_tests.rs:611-626", op="index_select",
                  x=list(range(1, 13)), shape=[4, 3], ids=[0, 2, 3], dim=0,
                  expected=[1, 2, 3, 7, 8, 9, 10, 11, 12], expected_shape=[3, 3]))
    c.append(dict(name="index_select_2d_dim1", source="mimi-rs/tests/cuda_tests.rs:628-643", op="index_select",
                  x=list(range(1, 13)), shape=[3, 4], ids=[1, 3], dim=1,
                  expected=[2, 4, 6, 8, 10, 12], expected_shape=[3, 2]))
    c.append(dict(name="index_select_3d", source="mimi-rs/tests/cuda_tests.rs:645-665", op="index_select",
                  x=list(range(1, 25)), shape=[2, 3, 4], ids=[0, 2], dim=1,
                  expected=[1, 2, 3, 4, 9, 10, 11, 12, 13, 14, 15, 16, 21, 22, 23, 24], expected_shape=[2, 2, 4]))
    c.append(dict(name="index_select_dim0_repeat", source="mimi-rs/tests/tensor_tests.rs:121-137",
                  op="index_select", x=list(range(1, 13)), shape=[4, 3], ids=[1, 1, 0], dim=0,
                  expected=[4, 5, 6, 4, 5, 6, 1, 2, 3], expected_shape=[3, 3]))
    c.append(dict(name="index_select_dim1_2x4", source="mimi-rs/tests/tensor_tests.rs:139-150",
                  op="index_select", x=list(range(1, 9)), shape=[2, 4], ids=[0, 2], dim=1,
                  expected=[1, 3, 5, 7], expected_shape=[2, 2]))
    c.append(dict(name="index_select_3d_2x3x2", source="mimi-rs/tests/tensor_tests.rs:152-167",
                  op="index_select", x=list(range(1, 13)), shape=[2, 3, 2], ids=[0, 2], dim=1,
                  expected=[1, 2, 5, 6, 7, 8, 11, 12], expected_shape=[2, 2, 2]))
    c.append(dict(name="causality_mask", source="mimi-rs/tests/cuda_tests.rs:756-790", op="causality_mask",
                  shape=[1, 3, 4], fill=1.0, offset=0,
                  expected=[1, NEG_INF, NEG_INF, NEG_INF, 1, 1, NEG_INF, NEG_INF, 1, 1, 1, NEG_INF]))
    c.append(dict(name="causality_mask_with_offset", source="mimi-rs/tests/cuda_tests.rs:792-818",
                  op="causality_mask", shape=[1, 2, 4], fill=1.0, offset=2,
                  expected=[1, 1, 1, NEG_INF, 1, 1, 1, 1]))
    cos = [1, 1, 0, 0, -1, -1, 0, 0, 1, 1, 0.5, 0.5, 0, 0, 0, 0, 0, 0, 0, 0]
    sin = [0, 0, 1, 1, 0, 0, 0, 0, 0, 0, 0.866, 0.866, 0, 0, 0, 0, 0, 0, 0, 0]
    c.append(dict(name="rope_position_offset_pos0", source="mimi-rs/tests/cuda_tests.rs:1109-1158", op="rope",
                  x=[1, 2, 3, 4], shape=[1, 1, 1, 4], cos=cos, sin=sin, table_shape=[10, 2], pos=0,
                  expected=[1, 2, 3, 4], tol=1e-5))
    # The test asserts "not identity" at pos 1; its comment (cuda_tests.rs:1160-1164)
    # spells out the rotated values, which are asserted here.
    c.append(dict(name="rope_position_offset_pos1", source="mimi-rs/tests/cuda_tests.rs:1160-1173", op="rope",
                  x=[1, 2, 3, 4], shape=[1, 1, 1, 4], cos=cos, sin=sin, table_shape=[10, 2], pos=1,
                  expected=[-3, -4, 1, 2], tol=1e-5, not_identity=True))
    k = [i / 100.0 for i in range(1280)]
    c.append(dict(name="rope_identity_tables", source="mimi-rs/tests/cuda_tests.rs:1059-1076", op="rope",
                  x=k, shape=[1, 4, 5, 64], cos=[1.0] * 320, sin=[0.0] * 320, table_shape=[10, 32], pos=0,
                  expected=k, tol=1e-5, note="x is k.transpose(1,2).contiguous(); identity holds for any layout"))
    return c


def main():
    data = {"generator": "tests/golden/make_known_answers.py", "cases": cases()}
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {OUT} ({len(data['cases'])} cases)")


if __name__ == "__main__":
    main()
