"""Builds libxn_fused.so, the sm_100a fused layer-op library, in-tree.

Usage: python random-things_b200/build.py [--force] [--verbose]

Each csrc/*.cu file is compiled to an object with nvcc for sm_100a only, then
linked into one shared library next to this file. The C ABI it exports is
declared in include/xn_fused.h. Objects are rebuilt when their source or any
header is newer.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libxn_fused.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: the reference CPU backend never fuses a*b+c, so neither may the
# kernels (explicit __f*_rn intrinsics are used as well; CUDA's math functions
# use explicit fma internally and are unaffected).
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-fmad=false",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the fused-op library needs the CUDA toolkit to build")
    return cand


def host_compiler() -> list[str]:
    # A gcc wrapper earlier on PATH may lack parts of the toolchain; prefer the system one.
    for c in ("/usr/bin/g++",):
        if Path(c).exists():
            return ["-ccbin", c]
    return []


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _newest(paths: list[Path]) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    hdr_time = _newest(headers())
    objs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
            continue
        cmd = [nvcc, *host_compiler(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}",
               "-c", str(src), "-o", str(obj)]
        # The exported C ABI keeps default visibility through XN_API in the sources.
        if ptxas_verbose:
            cmd.insert(-4, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _newest(objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *host_compiler(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs),
               "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
