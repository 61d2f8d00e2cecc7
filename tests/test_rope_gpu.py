"""GPU parity: RoPE (half-split and interleaved) against the oracle's
restatement of cpu_backend.rs:359-422. The kernel rounds at every point the
reference rounds, so results are required to be bit-exact for every dtype."""
import numpy as np
import pytest
import torch

from helpers import from_device, randn, rng, to_device, to_storage

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "bf16", "f16"]
# (b, h, t, d, pos, max_pos): benchmark config 1 (Q/K 16x128 heads), config 2
# (8x64, 250 frames), config 3 decode (t=1 at a position), config 4-like heads,
# and ragged half-dims that take the scalar path.
SHAPES = [
    (1, 16, 512, 128, 0, 512),
    (4, 8, 250, 64, 0, 8192),
    (16, 16, 1, 64, 137, 256),
    (2, 8, 64, 128, 5, 4096),
    (2, 3, 7, 6, 2, 16),
    (1, 2, 5, 4, 0, 10),
    (1, 5, 3, 2, 1, 4),
]


def _case(seed, b, h, t, d, max_pos, dtype, variant):
    r = rng(seed)
    x = to_storage(randn(r, (b, h, t, d)), dtype)
    return x


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b,h,t,d,pos,max_pos", SHAPES)
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_bhtd_bit_exact(oracle, xn, cuda, dtype, b, h, t, d, pos, max_pos, interleaved):
    x = _case(b * h * t + d, b, h, t, d, max_pos, dtype, interleaved)
    cos, sin = oracle.rope_tables(d, max_pos, 10000.0, dtype, "mimi")
    ref = oracle.rope(x, cos, sin, pos, dtype, interleaved=interleaved)
    X, C, S = (to_device(a, dtype, cuda) for a in (x, cos, sin))
    Y = xn.rope_i(X, C, S, pos) if interleaved else xn.rope(X, C, S, pos)
    assert np.array_equal(from_device(Y, dtype), ref)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b,h,t,d,pos,max_pos", SHAPES[:5])
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_bthd_layout(oracle, xn, cuda, dtype, b, h, t, d, pos, max_pos, interleaved):
    """[B,T,H,D] input == transpose -> reference rope -> transpose back
    (pocket_tts/src/rope.rs:42-48), without the copies."""
    x = _case(b + h + t + d, b, h, t, d, max_pos, dtype, interleaved)
    cos, sin = oracle.rope_tables(d, max_pos, 10000.0, dtype, "mimi")
    ref = oracle.rope(x, cos, sin, pos, dtype, interleaved=interleaved)  # x is [B,H,T,D]
    x_bthd = np.ascontiguousarray(np.swapaxes(x, 1, 2))
    ref_bthd = np.ascontiguousarray(np.swapaxes(ref, 1, 2))
    X, C, S = (to_device(a, dtype, cuda) for a in (x_bthd, cos, sin))
    Y = (xn.rope_i if interleaved else xn.rope)(X, C, S, pos, layout="bthd")
    assert np.array_equal(from_device(Y, dtype), ref_bthd)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rope_qk_one_launch(oracle, xn, cuda, dtype):
    """Q with 32 heads and K with 8 heads (config 4 GQA shape, shortened T)."""
    r = rng(7)
    b, t, d, pos = 2, 96, 128, 3
    q = to_storage(randn(r, (b, 32, t, d)), dtype)
    k = to_storage(randn(r, (b, 8, t, d)), dtype)
    cos, sin = oracle.rope_tables(d, 4096, 500000.0, dtype, "llama")
    C, S = to_device(cos, dtype, cuda), to_device(sin, dtype, cuda)
    for inter in (False, True):
        Qo, Ko = xn.rope_qk(to_device(q, dtype, cuda), to_device(k, dtype, cuda), C, S, pos, interleaved=inter)
        assert np.array_equal(from_device(Qo, dtype), oracle.rope(q, cos, sin, pos, dtype, interleaved=inter))
        assert np.array_equal(from_device(Ko, dtype), oracle.rope(k, cos, sin, pos, dtype, interleaved=inter))


def test_rope_inplace_and_errors(oracle, xn, cuda):
    r = rng(8)
    x = randn(r, (2, 4, 9, 64))
    cos, sin = oracle.rope_tables(64, 16, 10000.0, "f32", "mimi")
    X, C, S = (to_device(a, "f32", cuda) for a in (x, cos, sin))
    xn.rope_(X, X, C, S, 7)
    assert np.array_equal(from_device(X, "f32"), oracle.rope(x, cos, sin, 7, "f32"))
    with pytest.raises(xn.XnError, match="position out of range"):
        xn.rope(X, C, S, 8)  # 8 + 9 > 16
    with pytest.raises(xn.XnError, match="even d"):
        xn.rope(torch.zeros(1, 1, 2, 3, device=cuda), torch.zeros(4, 1, device=cuda),
                torch.zeros(4, 1, device=cuda), 0)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("b,t,h,d,pos", [(4, 250, 8, 64, 0), (16, 1, 16, 64, 77), (2, 9, 3, 6, 1)])
def test_rope_qk_packed_projection(oracle, xn, cuda, dtype, interleaved, b, t, h, d, pos):
    """Q and K read in place from the packed QKV projection equal the reference's
    narrow -> reshape -> transpose -> contiguous -> rope_i (mimi.rs:1332-1351)."""
    r = rng(b * t + h * d + pos)
    qkv = to_storage(randn(r, (b, t, 3 * h * d)), dtype)
    cos, sin = oracle.rope_tables(d, pos + t + 3, 10000.0, dtype, "mimi")
    ref = []
    for part in range(2):
        x = np.ascontiguousarray(qkv[..., part * h * d:(part + 1) * h * d].reshape(b, t, h, d).swapaxes(1, 2))
        y = oracle.rope(x, cos, sin, pos, dtype, interleaved=interleaved)
        ref.append(np.ascontiguousarray(y.swapaxes(1, 2)))
    Q, K = xn.rope_qk_packed(to_device(qkv, dtype, cuda), h, to_device(cos, dtype, cuda), to_device(sin, dtype, cuda),
                             pos, interleaved=interleaved)
    assert np.array_equal(from_device(Q, dtype), ref[0])
    assert np.array_equal(from_device(K, dtype), ref[1])
