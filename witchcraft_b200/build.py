"""Builds the native library `witchcraft_b200/libwc_t5cuda.so` in-tree.

Every CUDA translation unit is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`); the host C++ parts with g++.
The library links the CUDA runtime statically and reaches the driver's
cuTensorMapEncodeTiled through cudaGetDriverEntryPointByVersion, so it needs
no libcuda at link time and no torch at all.

Usage: python -m witchcraft_b200.build   (or witchcraft_b200.build.build())
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libwc_t5cuda.so")
BUILD_DIR = os.path.join(HERE, "_build")

CUDA_SOURCES = ["gemm_q4k.cu", "gemm2_q4k.cu", "gemv_q4k.cu", "attention_tc.cu", "attention_small.cu", "elementwise.cu", "runtime.cu", "codec.cu", "index.cu", "query.cu"]
CXX_SOURCES = ["t5_host.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(os.path.dirname(HERE), "include")
    headers += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    objs = []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            extra = os.environ.get("WC_EXTRA_NVCC_FLAGS", "").split()
            out = _run([nvcc, *ARCH, *extra, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                        "--expt-relaxed-constexpr", "-c", s, "-o", o])
            if verbose:
                print(out)
    for src in CXX_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-I/usr/local/cuda/include", "-c", s, "-o", o])
    if force or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o", LIB, *objs])
    return LIB


def build_oracle() -> str:
    """Builds the CPU oracle (test infrastructure) with its Makefile."""
    d = os.path.join(os.path.dirname(HERE), "oracle")
    _run(["make", "-C", d, "CC=gcc"])
    return os.path.join(d, "liboracle.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
