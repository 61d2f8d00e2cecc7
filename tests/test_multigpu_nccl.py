"""Row-sharded execution on several GPUs with NCCL: each rank runs the fused
kernels on its xn_shard_rows block and the optional all-gather reassembles the
output on every rank, which must equal the single-GPU result bit for bit.
Runs as child processes, one per GPU (skipped with fewer than 2 GPUs)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path

    import torch.distributed as dist

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "random-things_b200"))
    import xn_fused as xn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        rows, cols = 1000, 4096
        x = torch.randn(rows, cols, device=dev, generator=g).to(torch.bfloat16)
        br = torch.randn(rows, cols, device=dev, generator=g).to(torch.bfloat16)
        a = (torch.randn(cols, device=dev, generator=g) * 0.02 + 1).to(torch.bfloat16)
        full_y, full_h = xn.rms_norm_residual(x, br, a, 1e-5)
        begin, count = xn.shard_rows(rows, world, rank)
        y, h = xn.rms_norm_residual(x[begin:begin + count], br[begin:begin + count], a, 1e-5)
        gy = xn.all_gather_rows(y, rows)
        gh = xn.all_gather_rows(h, rows)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(gy, full_y) and torch.equal(gh, full_h)), count))
    finally:
        dist.destroy_process_group()


def test_row_sharded_norm_with_nccl_gather():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results), results
    assert sum(c for _, _, c in results) == 1000
