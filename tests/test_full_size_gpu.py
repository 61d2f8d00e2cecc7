"""Whole-tensor checks at the full sizes of the benchmark configurations,
where running the CPU oracle over every element would take too long.

The per-element steps whose results depend on a transcendental function
(SiLU, the softmax's exp) come from the oracle as lookup tables over every
bf16 input. torch on the GPU then evaluates the rest of the reference's op
sequence, where a torch bf16 operation rounds exactly as the reference's T
arithmetic does (one rounding of the f32 result: cpu_backend.rs:224-258 for
add/sub/mul, :359-392 for RoPE, :624-645 for the gather). Where only the
order of an f32 row sum differs (RMSNorm, the softmax denominator), the bound
is one ulp, the fused-op tolerance of the smaller oracle comparisons.

torch is the checker here, never the thing measured: every output comes
from the sm_100a kernels through the C ABI."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CHUNK = 1 << 27  # elements per chunk of the torch-side references


def _key(x: torch.Tensor) -> torch.Tensor:
    """Monotone integer key of bf16 values (finite or inf): consecutive keys
    are consecutive bf16 values, so key differences count ulps."""
    v = x.view(torch.int16).to(torch.int32)
    mag = v & 0x7FFF
    return torch.where(v < 0, -mag, mag)


def _max_ulp(a: torch.Tensor, b: torch.Tensor) -> int:
    return int((_key(a) - _key(b)).abs().max())


def _table(oracle, op: str) -> torch.Tensor:
    """The oracle's bf16 result of `op` for every 16-bit input pattern."""
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    return torch.from_numpy(oracle.unary(bits, op, "bf16").view(np.int16).copy())


def _lookup(table: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    return table[x.view(torch.int16).long() & 0xFFFF].view(torch.bfloat16)


def _row_chunks(rows: int, cols: int):
    step = max(1, CHUNK // cols)
    for r0 in range(0, rows, step):
        yield r0, min(rows, r0 + step)


@pytest.fixture(scope="module")
def config4_step(xn, cuda):
    import bench

    wl = bench.LlamaPrefillOps(torch, xn, cuda, bench.CFG, seed=77)
    wl.step()
    torch.cuda.synchronize()
    yield wl
    del wl
    torch.cuda.empty_cache()


def test_config4_gather_rope_residual(config4_step):
    """Benchmark config 4, every element: the gather of 32768 ids from the
    128256 x 4096 table equals torch's indexing byte for byte; RoPE of Q
    [8, 32, 4096, 128] and K [8, 8, 4096, 128] equals the reference's sequence
    T(T(x1 c) - T(x2 s)), T(T(x1 s) + T(x2 c)); the residual h equals T(x + b)."""
    import bench

    wl = config4_step
    assert torch.equal(wl.x, wl.table[wl.ids.long()])
    assert torch.equal(wl.h, wl.x + wl.attn_out)
    half = bench.CFG["head_dim"] // 2
    c, s = wl.cos[None, None], wl.sin[None, None]  # [1, 1, S, D/2]
    for src, out in ((wl.q, wl.qo), (wl.k, wl.ko)):
        for b in range(src.shape[0]):
            x1, x2 = src[b : b + 1, ..., :half], src[b : b + 1, ..., half:]
            ref = torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)
            assert torch.equal(out[b : b + 1], ref), f"rope differs in batch element {b}"


def test_config4_rms_norms(config4_step):
    """Both RMSNorms of the step, every element within one bf16 ulp of the
    reference's expression x / sqrt(sum(x^2) / n + eps) * alpha, evaluated in
    f32 and rounded once (cpu_backend.rs:691-709): the two differ only in the
    order of the f32 row sum."""
    import bench

    wl, eps = config4_step, bench.CFG["eps"]
    for x, alpha, y in ((wl.x, wl.alpha1, wl.y1), (wl.h, wl.alpha2, wl.y2)):
        for r0, r1 in _row_chunks(*x.shape):
            xf = x[r0:r1].float()
            m = torch.sqrt((xf * xf).sum(dim=-1, keepdim=True) / x.shape[1] + eps)
            ref = (xf / m * alpha.float()).to(torch.bfloat16)
            assert _max_ulp(y[r0:r1], ref) <= 1, f"rows {r0}..{r1}"


def test_config4_swiglu_bit_exact(oracle, config4_step):
    """SwiGLU on [32768, 14336], every element bit for bit: T(silu(g) * u) with
    silu(g) from the oracle's SiLU (cpu_backend.rs:213-215, llama.rs:256-263)
    over every bf16 input and the product rounded once by torch."""
    wl = config4_step
    silu = _table(oracle, "silu").to(wl.gate.device)
    for r0, r1 in _row_chunks(*wl.gate.shape):
        ref = _lookup(silu, wl.gate[r0:r1]) * wl.up[r0:r1]
        assert torch.equal(wl.act[r0:r1], ref), f"rows {r0}..{r1}"


def test_rvq_decode_bit_exact(xn, cuda):
    """The RVQ gather-sum against torch's (((E0[c0] + E1[c1]) + E2[c2]) + ...),
    each add rounded once as the reference's T add (mimi.rs:1730-1744), bit for
    bit: config 2's shape (batch 4, 8 codebooks of 2048 x 256, 250 frames) and
    one sequence of 1M frames."""
    g = torch.Generator(device=cuda).manual_seed(5)
    books = [torch.randn((2048, 256), device=cuda, generator=g).to(torch.bfloat16) for _ in range(8)]
    for batch, frames in ((4, 250), (1, 1 << 20)):
        codes = torch.randint(0, 2048, (batch, 8, frames), device=cuda, generator=g, dtype=torch.int64)
        got = xn.rvq_decode_sum(books, codes, out_layout="btd")
        ref = books[0][codes[:, 0]]
        for q in range(1, 8):
            ref = ref + books[q][codes[:, q]]
        assert torch.equal(got, ref), f"batch {batch}, {frames} frames"


@pytest.mark.parametrize("rows,cols", [(1 << 20, 1024), (65536, 16384)])
def test_softmax_config5_largest(oracle, xn, cuda, rows, cols):
    """Config 5's largest bf16 softmax points, every element within one ulp of
    the reference's sequence (cpu_backend.rs:667-689): m = max, e = T(exp(T(x -
    m))) from the oracle's exp over every bf16 input, s = the f32 sum of e, y =
    T(e / s). Only the order of the f32 sum differs."""
    g = torch.Generator(device=cuda).manual_seed(6)
    x = torch.randn((rows, cols), device=cuda, generator=g).to(torch.bfloat16)
    y = xn.softmax(x)
    exp = _table(oracle, "exp").to(cuda)
    for r0, r1 in _row_chunks(rows, cols):
        xf = x[r0:r1].float()
        arg = (xf - xf.amax(dim=-1, keepdim=True)).to(torch.bfloat16)  # exact difference, rounded once
        e = _lookup(exp, arg).float()
        ref = (e / e.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
        assert _max_ulp(y[r0:r1], ref) <= 1, f"rows {r0}..{r1}"
    del x, y
    torch.cuda.empty_cache()
