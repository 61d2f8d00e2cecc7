"""Builds the C++ port of the reference's CUDA known-answer tests
(tests/cpp/test_backend.cpp, on the C++ Backend mirror) and, on a GPU, runs it."""
import os
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "random-things_b200"
EXE = REPO / "tests" / "cpp" / "_build" / "test_backend"


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    return "nvcc"


def build_harness() -> Path:
    EXE.parent.mkdir(parents=True, exist_ok=True)
    cmd = [_nvcc(), "-ccbin", "/usr/bin/g++", "-std=c++17", "-O2", f"-I{REPO / 'include'}", f"-I{PKG / 'host'}",
           str(REPO / "tests" / "cpp" / "test_backend.cpp"), "-o", str(EXE), f"-L{PKG}", "-lxn_fused",
           f"-Xlinker=-rpath={PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return EXE


def test_cpp_harness_builds(xn):
    assert build_harness().exists()


@pytest.mark.gpu
def test_cpp_known_answers_on_gpu(xn, cuda):
    exe = build_harness()
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 failed" in out.stdout
