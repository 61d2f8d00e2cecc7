"""Maximum sizes: each op over more than 2^31 elements (4.3 GB per bf16
tensor), so any 32-bit element index would overflow. Rows are independent,
so only the last rows are compared with the oracle."""
import numpy as np
import pytest
import torch

from helpers import assert_close, from_device

pytestmark = pytest.mark.gpu

COLS = 4096
ROWS = (1 << 31) // COLS + 64  # 2^31 + 64 * 4096 elements
TAIL = 8


def _bits(t: torch.Tensor) -> np.ndarray:
    return from_device(t, "bf16")


@pytest.fixture(scope="module")
def big(cuda):
    g = torch.Generator(device=cuda).manual_seed(31)
    x = torch.empty((ROWS, COLS), dtype=torch.bfloat16, device=cuda)
    for r0 in range(0, ROWS, 65536):  # fill in chunks to bound the f32 temporary
        r1 = min(ROWS, r0 + 65536)
        x[r0:r1] = torch.randn((r1 - r0, COLS), device=cuda, generator=g).to(torch.bfloat16)
    yield x
    del x
    torch.cuda.empty_cache()


def test_rms_norm_past_2_31_elements(oracle, xn, cuda, big):
    w = (torch.randn(COLS, device=cuda) * 0.02 + 1).to(torch.bfloat16)
    y = xn.rms_norm(big, w, 1e-5)
    ref = oracle.rms_norm(_bits(big[-TAIL:]), _bits(w), 1e-5, "bf16")
    assert_close(_bits(y[-TAIL:]), ref, "bf16", "rms_norm tail")
    del y


def test_softmax_past_2_31_elements(oracle, xn, cuda, big):
    y = xn.softmax(big)
    assert_close(_bits(y[-TAIL:]), oracle.softmax(_bits(big[-TAIL:]), "bf16"), "bf16", "softmax tail")
    del y


def test_swiglu_and_gather_past_2_31_elements(oracle, xn, cuda, big):
    up = big.flip(0)  # a second operand of the same size, rows in reverse order
    y = xn.swiglu(big, up.contiguous())
    ref = oracle.swiglu(_bits(big[-TAIL:]), _bits(up[-TAIL:]), "bf16")
    assert_close(_bits(y[-TAIL:]), ref, "bf16", "swiglu tail")
    del y, up
    torch.cuda.empty_cache()
    ids = torch.arange(ROWS - 1, -1, -1, dtype=torch.int64, device=cuda)  # reverse every row
    g = xn.index_select(big, ids, 0)
    assert torch.equal(g[:TAIL], big[-TAIL:].flip(0)) and torch.equal(g[-TAIL:], big[:TAIL].flip(0))
