"""Concurrent use of the library from many host threads (the situation of the
reference's mimi-rs/examples/cuda_thread_test.rs: 32 threads, each with its
own device handle, running different ops). Each thread launches on its own
CUDA stream; every result must equal the same op run alone, bit for bit."""
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops(xn, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)

    def rnd(*shape, std=1.0):
        return (torch.randn(shape, device=dev, generator=g) * std).to(torch.bfloat16)

    x, br, w = rnd(256, 1024), rnd(256, 1024), rnd(1024, std=0.02) + 1
    q, cos, sin = rnd(2, 8, 64, 64), rnd(128, 32), rnd(128, 32)
    s = rnd(64, 512, std=2.0)
    gate, up = rnd(128, 2048), rnd(128, 2048)
    table, ids = rnd(512, 256), torch.randint(0, 512, (300,), device=dev, generator=g)

    def run():
        y, h = xn.rms_norm_residual(x, br, w, 1e-5)
        return [y, h, xn.rope_i(q, cos, sin, 7), xn.softmax(s), xn.swiglu(gate, up), xn.index_select(table, ids, 0)]

    return run


def test_threads_on_own_streams_match_serial(xn, cuda):
    n_threads, reps = 8, 10
    runners = [_ops(xn, 100 + i, cuda) for i in range(n_threads)]
    expected = [r() for r in runners]
    torch.cuda.synchronize()
    results, errors = [None] * n_threads, []
    barrier = threading.Barrier(n_threads)

    def worker(i):
        try:
            stream = torch.cuda.Stream(cuda)
            with torch.cuda.stream(stream):
                barrier.wait()
                for _ in range(reps):
                    out = runners[i]()
                stream.synchronize()
            results[i] = out
        except Exception as e:  # reported below
            errors.append(repr(e))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(n_threads)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for i in range(n_threads):
        for got, want in zip(results[i], expected[i]):
            assert torch.equal(got, want), f"thread {i}"
