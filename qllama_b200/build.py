"""Builds libqllama_attn.so in-tree with nvcc for sm_100a."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqllama_attn.so")
BENCH_LIB = os.path.join(HERE, "libqllama_bench.so")
SOURCES = ["ql_api.cu", "ql_kernels.cu", "ql_prefill_tc.cu", "ql_model.cu", "ql_gguf.cpp"]
HEADERS = ["ql_device.cuh", "ql_kernels.cuh", "ql_append.cuh", "ql_internal.h",
           os.path.join("..", "..", "include", "qllama_model.h"), os.path.join("..", "..", "include", "qllama_attn.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-cudart", "static", "-ldl",
]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(os.path.join(CSRC, d)) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    nvcc = os.environ.get("NVCC", "nvcc")
    if force or _stale(LIB, SOURCES + HEADERS):
        cmd = [nvcc, *NVCC_FLAGS, "-o", LIB, *[os.path.join(CSRC, s) for s in SOURCES]]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True, cwd=CSRC)
    # Native driver of whole prefill+decode jobs for bench.py (links the library).
    if force or _stale(BENCH_LIB, ["bench_driver.cpp", HEADERS[-1]]) or \
            os.path.getmtime(BENCH_LIB) < os.path.getmtime(LIB):
        cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-o", BENCH_LIB,
               os.path.join(CSRC, "bench_driver.cpp"), "-L" + HERE, "-lqllama_attn",
               "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True, cwd=CSRC)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
