"""GPU parity for the integer-indexed gathers (bit-exact): index_select with
device ids (cpu_backend.rs:624-645) and the fused RVQ decode sum
(mimi.rs:1627-1744)."""
import numpy as np
import pytest
import torch

from helpers import from_device, randn, rng, to_device, to_storage

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16", "i64", "u8"])
@pytest.mark.parametrize("shape,dim,n_ids", [((1000, 256), 0, 300), ((50, 3), 0, 17), ((4, 9, 5), 1, 6),
                                             ((2, 8, 64, 128), 1, 32), ((3, 4), 1, 2), ((100, 4096), 0, 1)])
@pytest.mark.parametrize("id_dtype", [np.int64, np.int32])
def test_index_select(oracle, xn, cuda, dtype, shape, dim, n_ids, id_dtype):
    r = rng(sum(shape) + n_ids)
    if dtype in ("f32", "bf16", "f16"):
        x = to_storage(randn(r, shape), dtype)
        X = to_device(x, dtype, cuda)
    else:
        npdt = np.int64 if dtype == "i64" else np.uint8
        x = r.integers(0, 200, size=shape).astype(npdt)
        X = torch.from_numpy(x).to(cuda)
    ids = r.integers(0, shape[dim], size=n_ids)
    ref = oracle.index_select(x, ids.astype(np.uint32), dim)
    ids_t = torch.from_numpy(ids.astype(id_dtype)).to(cuda)
    Y = xn.index_select(X, ids_t, dim)
    got = from_device(Y, dtype) if dtype in ("f32", "bf16", "f16") else Y.cpu().numpy()
    assert np.array_equal(got, ref)


def test_index_select_config4_embedding(oracle, xn, cuda):
    """Config 4 embedding gather, shortened: [128256, 4096] bf16, u32-like ids."""
    r = rng(4)
    vocab, hidden, n = 128256, 4096, 2048
    table = torch.randn(vocab, hidden, device=cuda, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
    ids = r.integers(0, vocab, size=n)
    Y = xn.index_select(table, torch.from_numpy(ids.astype(np.int32)).to(cuda), 0)
    assert torch.equal(Y, table[torch.from_numpy(ids).to(cuda)])


def test_index_select_out_of_range_flag(xn, cuda):
    X = torch.arange(20, dtype=torch.float32, device=cuda).view(5, 4)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ids = torch.tensor([1, 7, -1, 4], dtype=torch.int64, device=cuda)
    Y = xn.index_select(X, ids, 0, err_flag=err)
    assert int(err.item()) == 1
    assert torch.equal(Y[0], X[1]) and torch.equal(Y[3], X[4])
    assert torch.all(Y[1] == 0) and torch.all(Y[2] == 0)
    # Host ids are checked on the host, like the reference (tensor.rs:170-176).
    with pytest.raises(xn.XnError, match="out of bounds"):
        xn.index_select(X, [0, 5], 0)
    # Empty id list.
    assert xn.index_select(X, torch.zeros(0, dtype=torch.int64, device=cuda), 0).shape == (0, 4)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("layout", ["bct", "btd"])
@pytest.mark.parametrize("b,q,t,bins,dim", [(4, 8, 250, 2048, 256), (1, 1, 1, 4, 8), (2, 3, 37, 16, 6),
                                            (3, 32, 65, 64, 64), (1, 2, 5, 8, 1100)])
def test_rvq_decode_sum(oracle, xn, cuda, dtype, layout, b, q, t, bins, dim):
    r = rng(b * q * t + dim)
    books = [to_storage(randn(r, (bins, dim)), dtype) for _ in range(q)]
    codes = r.integers(0, bins, size=(b, q, t), dtype=np.int64)
    ref = oracle.rvq_decode(books, codes, dtype, layout)
    Y = xn.rvq_decode_sum([to_device(cb, dtype, cuda) for cb in books], torch.from_numpy(codes).to(cuda),
                          out_layout=layout)
    assert np.array_equal(from_device(Y, dtype), ref)


def test_rvq_bad_code_flag(xn, cuda):
    books = [torch.ones(4, 8, device=cuda), torch.full((4, 8), 2.0, device=cuda)]
    codes = torch.tensor([[[0, 1, 2], [3, 9, 1]]], dtype=torch.int64, device=cuda)  # [1, 2, 3]
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    Y = xn.rvq_decode_sum(books, codes, out_layout="btd", err_flag=err)
    assert int(err.item()) == 1
    assert torch.all(Y[0, 0] == 3) and torch.all(Y[0, 1] == 1) and torch.all(Y[0, 2] == 3)


@pytest.mark.parametrize("dtype,row", [("bf16", 1024), ("bf16", 4096), ("f32", 4096), ("bf16", 24576),
                                       ("bf16", 256), ("f32", 64), ("bf16", 24), ("f32", 12)])
def test_index_select_bad_ids_in_every_row_shape(oracle, xn, cuda, dtype, row):
    """Rows of 48 B to 48 KB (several rows per warp item, one item per row,
    several items per row); bad ids interleaved with good ones give zero rows
    and bit 1 of the flag, the other rows stay exact."""
    r = rng(row)
    table = to_storage(randn(r, (300, row)), dtype)
    ids = r.integers(0, 300, size=777)
    ids[::50] = -3
    ids[7::61] = 300
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    Y = from_device(xn.index_select(to_device(table, dtype, cuda), torch.from_numpy(ids).to(cuda), 0,
                                    err_flag=err), dtype)
    assert int(err.item()) == 1
    bad = (ids < 0) | (ids >= 300)
    good_ids = np.where(bad, 0, ids).astype(np.uint32)
    ref = oracle.index_select(table, good_ids, 0)
    assert np.array_equal(Y[~bad], ref[~bad])
    assert np.all(Y[bad] == 0)
