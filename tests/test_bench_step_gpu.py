"""Parity of the exact step `bench.py` times (benchmark config 4, bf16): the
LlamaPrefillOps workload at its full size (32768 token rows, the 128256 x 4096
embedding table, Q [8, 32, 4096, 128] / K [8, 8, 4096, 128], SwiGLU on
[32768, 14336]), run once through the same code path and launch shapes as
the timed region, then checked on 256 sampled rows of every output against
the oracle (the reference CPU backend's op sequence: index_select,
rms_norm, rope, add + rms_norm, silu + mul; cpu_backend.rs:359-392,624-645,
691-709,213-258). The gather and RoPE are bit-exact; the norms and SwiGLU
within the tolerance of helpers.assert_close."""
import numpy as np
import pytest
import torch

from helpers import assert_close, from_device

pytestmark = pytest.mark.gpu

SAMPLE = 256


def test_bench_config4_step_matches_oracle(oracle, xn, cuda):
    import bench

    wl = bench.LlamaPrefillOps(torch, xn, cuda, bench.CFG, seed=1234)
    wl.step()
    torch.cuda.synchronize()
    c = bench.CFG
    r = np.random.default_rng(42)
    rows = np.sort(r.choice(wl.rows, SAMPLE, replace=False))
    idx = torch.from_numpy(rows).to(cuda)

    def take(t):
        return from_device(t.index_select(0, idx), "bf16")

    x = take(wl.x)
    ids = wl.ids.index_select(0, idx).cpu().numpy().astype(np.uint32)
    # 1. embedding gather: the sampled output rows are the table rows of their ids, bit for bit.
    table_rows = from_device(wl.table.index_select(0, torch.from_numpy(ids.astype(np.int64)).to(cuda)), "bf16")
    ref_x = oracle.index_select(table_rows, np.arange(SAMPLE, dtype=np.uint32), 0)
    assert np.array_equal(x, ref_x), "embedding gather differs"
    # 2. RMSNorm.
    a1, a2 = from_device(wl.alpha1, "bf16"), from_device(wl.alpha2, "bf16")
    assert_close(take(wl.y1), oracle.rms_norm(x, a1, c["eps"], "bf16"), "bf16", "rms_norm config4-step")
    # 4. residual + RMSNorm: h bit-exact, y2 within one ulp.
    ref_y2, ref_h = oracle.rms_norm_residual(x, take(wl.attn_out), a2, c["eps"], "bf16")
    assert np.array_equal(take(wl.h), ref_h), "residual output differs"
    assert_close(take(wl.y2), ref_y2, "bf16", "rms_norm_residual config4-step")
    # 5. SwiGLU on the sampled token rows.
    assert_close(take(wl.act), oracle.swiglu(take(wl.gate), take(wl.up), "bf16"), "bf16", "swiglu config4-step")
    # 3. RoPE: 256 sampled (b, h, t) rows of Q and of K, bit-exact.
    cos, sin = from_device(wl.cos, "bf16"), from_device(wl.sin, "bf16")
    for name, src, dst in (("q", wl.q, wl.qo), ("k", wl.k, wl.ko)):
        B, H, S, D = src.shape
        flat = r.choice(B * H * S, SAMPLE, replace=False)
        b, rem = np.divmod(flat, H * S)
        h, t = np.divmod(rem, S)
        bi, hi, ti = (torch.from_numpy(a).to(cuda) for a in (b, h, t))
        got = from_device(dst[bi, hi, ti], "bf16")
        inp = from_device(src[bi, hi, ti], "bf16")
        for i in range(SAMPLE):
            ref = oracle.rope(inp[i].reshape(1, 1, 1, D), cos, sin, int(t[i]), "bf16")
            assert np.array_equal(got[i], ref.reshape(D)), f"rope {name} differs at (b, h, t) = {b[i], h[i], t[i]}"
