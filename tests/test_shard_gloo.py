"""Row-sharded execution across ranks, on CPU with the gloo backend
(world_size 2 and 3): every rank takes its xn_shard_rows block, runs the
per-row op on it, and the optional all-gather reassembles the full output,
which must equal the unsharded result. The per-row op is the oracle's
RMSNorm (the host-side plan and gather logic are what is under test; on GPUs
the same plan feeds the CUDA kernels and the gather runs over NCCL)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, cols, q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    for p in (repo / "random-things_b200", repo / "oracle"):
        sys.path.insert(0, str(p))
    import xn_fused
    import xn_oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = np.random.default_rng(0)
        x = r.standard_normal((rows, cols), dtype=np.float32)
        a = r.standard_normal(cols, dtype=np.float32) * np.float32(0.02) + np.float32(1)
        begin, count = xn_fused.shard_rows(rows, world, rank)
        local = xn_oracle.rms_norm(np.ascontiguousarray(x[begin:begin + count]), a, 1e-5, "f32")
        full = xn_fused.all_gather_rows(torch.from_numpy(local), rows)
        ok = np.array_equal(full.numpy(), xn_oracle.rms_norm(x, a, 1e-5, "f32"))
        q.put((rank, ok, count))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows", [(2, 37), (3, 10), (2, 1)])
def test_row_sharding_with_gather(world, rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, 16, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results)
    assert sum(c for _, _, c in results) == rows


def _dying_worker(rank, world, port, q):
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(repo / "random-things_b200"))
    import xn_fused

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    dist.barrier()
    if rank == world - 1:
        os._exit(3)  # this rank dies between steps, with nothing in flight
    try:
        xn_fused.all_gather_rows(torch.zeros((4, 8)), 4 * world)
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank must get an error, not hang
        q.put((rank, type(e).__name__))


def test_dead_rank_fails_the_gather_instead_of_hanging():
    """A rank that exits between steps: the surviving rank's next collective
    (the optional output all-gather) ends with an error within the process
    group's short timeout, instead of waiting for ever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and outcome != "no error", outcome
    assert procs[1].exitcode == 3
