"""CPU tests of the C ABI boundary: the library loads, exports exactly what
include/xn_fused.h declares, and rejects bad arguments with the documented
status codes before touching the GPU. Also checks that the Python mirror
raises on CPU tensors (there is no CPU fallback)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "xn_fused.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"XN_API\s+[\w\s\*]*?\b(xn_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    for name in ("xn_rms_norm", "xn_layer_norm", "xn_rope", "xn_rope_qk", "xn_unary", "xn_swiglu", "xn_softmax",
                 "xn_causality_mask", "xn_index_select", "xn_rvq_decode_sum", "xn_shard_rows", "xn_last_error",
                 "xn_abi_version"):
        assert name in syms


def test_library_exports_every_declared_symbol(xn):
    lib = xn.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in xn_fused.h but not exported"
        assert name in xn.SIGNATURES, f"{name} has no ctypes signature in xn_fused.py"
    assert lib.xn_abi_version() == 1


def _rc(xn, name, *args):
    return getattr(xn.lib(), name)(*args)


def test_argument_errors_without_gpu(xn):
    L = xn.lib()
    # eps must be positive (inplace_ops.rs:261)
    assert _rc(xn, "xn_rms_norm", 1, 1, 1, None, None, None, 4, 8, 0.0, 2, None) == xn.XN_E_INVALID
    assert "eps must be positive" in xn.last_error()
    # unsupported dtype
    assert _rc(xn, "xn_layer_norm", 1, 1, None, None, None, None, None, 4, 8, 1e-5, 1, 7, None) == xn.XN_E_DTYPE
    # layer scale without a branch
    assert _rc(xn, "xn_rms_norm", 1, 1, 1, None, 1, None, 4, 8, 1e-5, 2, None) == xn.XN_E_INVALID
    # rope: pos + t > max_pos (inplace_ops.rs:433-439) and odd d
    assert _rc(xn, "xn_rope", 1, 1, 1, 1, 1, 1, 5, 8, 6, 10, 0, 0, 2, None) == xn.XN_E_RANGE
    assert "position out of range" in xn.last_error()
    assert _rc(xn, "xn_rope", 1, 1, 1, 1, 1, 1, 5, 7, 0, 10, 0, 0, 2, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_rope", 1, 1, 1, 1, 1, 1, 5, 8, 0, 10, 0, 9, 2, None) == xn.XN_E_INVALID
    # unknown unary op, negative sizes
    assert _rc(xn, "xn_unary", 1, 1, 10, 5, 2, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_swiglu", 1, 1, 1, 4, 8, 4, 8, 2, None) == xn.XN_E_INVALID  # stride < cols
    assert _rc(xn, "xn_softmax", 1, 1, 6, 4, 1, 4, 0, 2, None) == xn.XN_E_INVALID  # t1 does not divide rows
    assert _rc(xn, "xn_index_select", 1, 1, 1, 0, 4, 1, 3, 2, 9, None, None) == xn.XN_E_DTYPE
    assert _rc(xn, "xn_index_select", 1, 1, 1, 0, -4, 1, 3, 2, 2, None, None) == xn.XN_E_INVALID
    tables = (ctypes.c_void_p * 1)(1)
    assert _rc(xn, "xn_rvq_decode_sum", 1, tables, 0, 1, 1, 1, 8, 4, 1, 2, None, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_rvq_decode_sum", 1, tables, 33, 1, 1, 1, 8, 4, 1, 2, None, None) == xn.XN_E_INVALID
    # decode: position past the tables, t > cap, odd head dim
    ap = "xn_kv_append_rope"
    assert _rc(xn, ap, 1, 1, 1, 1, 1, 1, 2, 4, 3, 64, 8, None, 10, 16, 1, 1, None, None) == xn.XN_E_RANGE
    assert _rc(xn, ap, 1, 1, 1, 1, 1, 1, 2, 4, 9, 64, 0, None, 100, 8, 1, 1, None, None) == xn.XN_E_INVALID
    assert _rc(xn, ap, 1, 1, 1, 1, 1, 1, 2, 4, 1, 63, 0, None, 100, 8, 1, 1, None, None) == xn.XN_E_INVALID
    at = "xn_attention_decode"
    # head dim outside {32, 64, 128}; context > cap; unknown mask mode; context above the shared-memory bound
    assert _rc(xn, at, 1, 1, 1, 1, 2, 4, 1, 48, 0, None, 16, 16, 0, 0.125, 1, None) == xn.XN_E_INVALID
    assert _rc(xn, at, 1, 1, 1, 1, 2, 4, 1, 64, 0, None, 16, 17, 0, 0.125, 1, None) == xn.XN_E_INVALID
    assert _rc(xn, at, 16, 16, 16, 16, 2, 4, 1, 64, 0, None, 16, 16, 3, 0.125, 1, None) == xn.XN_E_INVALID
    assert "unknown mask mode" in xn.last_error()
    assert _rc(xn, at, 1, 1, 1, 1, 2, 4, 1, 64, 0, None, 9000, 8193, 0, 0.125, 1, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_position_advance", None, 1, None) == xn.XN_E_INVALID
    # The fused decode step rotates at total (XN_MASK_ABSOLUTE): position 1000 is past 300 table rows.
    # XN_MASK_CACHE_LEN rotates at min(total, context) = 250, which is in range, so that call gets as
    # far as the null output pointer (every call here fails a host check before any launch).
    st = "xn_decode_attention_step"
    assert _rc(xn, st, None, 16, 16, 16, 16, 16, 1, 2, 1, 64, 1000, None, 300, 256, 250, xn.XN_MASK_ABSOLUTE, 0.125,
               1, 1, None, None) == xn.XN_E_RANGE
    assert _rc(xn, st, None, 16, 16, 16, 16, 16, 1, 2, 1, 64, 1000, None, 300, 256, 250, xn.XN_MASK_CACHE_LEN,
               0.125, 1, 1, None, None) == xn.XN_E_INVALID
    assert "null pointer" in xn.last_error()
    assert _rc(xn, st, None, 16, 16, 16, 16, 16, 1, 2, 1, 64, 0, None, 300, 256, 250, 3, 0.125, 1, 1, None,
               None) == xn.XN_E_INVALID
    # softmax with a status word: the checks of xn_softmax
    assert _rc(xn, "xn_softmax_status", 16, 16, -1, 4, 0, 1.0, 0, 1, 0, None, 2, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_softmax_status", 16, 16, 6, 4, 0, 1.0, 1, 4, 0, None, 2, None) == xn.XN_E_INVALID
    assert _rc(xn, "xn_softmax_status", 16, 16, 6, 4, 0, 1.0, 0, 1, 0, None, 9, None) == xn.XN_E_DTYPE
    assert L.xn_abi_version() == 1


def test_zero_sized_work_is_ok(xn):
    assert _rc(xn, "xn_rms_norm", None, None, None, None, None, None, 0, 8, 1e-5, 2, None) == xn.XN_OK
    assert _rc(xn, "xn_unary", None, None, 0, 0, 1, None) == xn.XN_OK
    assert _rc(xn, "xn_softmax", None, None, 0, 5, 0, 1, 0, 2, None) == xn.XN_OK
    assert _rc(xn, "xn_rope", None, None, None, None, 0, 4, 3, 8, 0, 10, 0, 0, 2, None) == xn.XN_OK
    assert _rc(xn, "xn_index_select", None, None, None, 0, 0, 1, 3, 2, 2, None, None) == xn.XN_OK
    assert xn.last_error() == ""


def test_shard_plan(xn):
    for rows, world in ((32768, 8), (10, 3), (3, 8), (0, 4), (7, 1)):
        spans = [xn.shard_rows(rows, world, r) for r in range(world)]
        covered = []
        for b, c in spans:
            covered.extend(range(b, b + c))
        assert covered == list(range(rows))
    with pytest.raises(xn.XnError):
        xn.shard_rows(10, 2, 2)


def test_python_mirror_checks(xn):
    x = torch.zeros(2, 3)
    with pytest.raises(xn.XnError, match="shape mismatch"):
        xn.rms_norm_(x, torch.zeros(3, 2), torch.ones(3), 1e-5)
    with pytest.raises(xn.XnError, match="eps must be positive"):
        xn.rms_norm_(x, x, torch.ones(3), 0.0)
    with pytest.raises(xn.XnError, match="no CPU path"):
        xn.rms_norm(x, torch.ones(3), 1e-5)
    with pytest.raises(xn.XnError, match="3D or 4D"):
        xn.apply_causality_mask(torch.zeros(3, 3), 0)


def test_error_messages_are_per_thread(xn):
    """xn_last_error() is thread-local: two threads that fail different checks
    at the same time each read back their own message (the C ABI is
    reentrant; status codes never depend on another thread's call)."""
    import threading

    lib = xn.lib()
    barrier = threading.Barrier(2)
    seen = {}

    def norm_thread():
        barrier.wait()
        for _ in range(200):
            rc = lib.xn_rms_norm(1, 1, 1, None, None, None, 4, 8, 0.0, 2, None)
            seen.setdefault("norm", set()).add((rc, xn.last_error().split(":")[0]))

    def rope_thread():
        barrier.wait()
        for _ in range(200):
            rc = lib.xn_rope(1, 1, 1, 1, 1, 1, 5, 8, 6, 10, 0, 0, 2, None)
            seen.setdefault("rope", set()).add((rc, xn.last_error().split(":")[0]))

    threads = [threading.Thread(target=norm_thread), threading.Thread(target=rope_thread)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert seen["norm"] == {(xn.XN_E_INVALID, "xn_rms_norm")}
    assert seen["rope"] == {(xn.XN_E_RANGE, "xn_rope")}


def test_every_kernel_waits_for_its_predecessor_first():
    """Launches allow programmatic dependent launch, so a kernel may start
    while the previous kernel of the stream drains. Every kernel must
    therefore begin with griddep_wait() (nothing read before it), and every
    launch must go through launch_k or another cudaLaunchKernelEx launcher that
    sets the same attribute (the softmax's cluster launch); no bare <<<...>>>
    launches."""
    import re
    from pathlib import Path

    csrc = Path(__file__).resolve().parents[1] / "random-things_b200" / "csrc"
    n_kernels = 0
    for f in sorted(csrc.glob("*.cu")):
        src = f.read_text()
        assert "<<<" not in src, f"{f.name}: bare <<<>>> launch"
        if "cudaLaunchKernelEx" in src:
            assert "cudaLaunchAttributeProgrammaticStreamSerialization" in src, f"{f.name}: launch without PDL"
        for m in re.finditer(r"__global__", src):
            body = src[src.index("{", m.end()) + 1:].lstrip()
            assert body.startswith("griddep_wait();"), f"{f.name}: kernel at offset {m.start()} does not wait first"
            n_kernels += 1
    assert n_kernels >= 19
