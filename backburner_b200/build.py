"""Builds libpacuda.so (the sm_100a kernels behind include/pa_cuda.h) in the package directory.

    python -m backburner_b200.build            # build if any source is newer than the library
    python -m backburner_b200.build --force    # rebuild
    python -m backburner_b200.build --verbose  # also print ptxas register / spill / shared-memory usage
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libpacuda.so")
SOURCES = ["pa_cuda.cu"]
GENCODE = "arch=compute_100a,code=sm_100a"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libpacuda.so")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "pa_cuda.h"))
    return files


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not verbose and not needs_build():
        return LIB
    cmd = [
        _nvcc(), "-gencode", GENCODE, "-lineinfo", "-O3", "-std=c++17",
        "--shared", "-Xcompiler", "-fPIC",
        "-I", INCLUDE, "-I", CSRC,
        "-o", LIB + ".tmp",
    ] + [os.path.join(CSRC, s) for s in SOURCES] + ["-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
