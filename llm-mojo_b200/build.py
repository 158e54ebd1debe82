"""Builds libmoe_b200.so in-tree with nvcc for sm_100a (B200).

    python llm-mojo_b200/build.py [--verbose]

The library is plain CUDA C++ behind the extern "C" ABI of include/moe_b200.h;
no PyTorch headers are involved, so any host language can load it.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmoe_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

SOURCES = ["moe_abi.cu", "moe_kernels.cu", "moe_tc.cu", "moe_tc_stream.cu", "moe_route.cu", "moe_gemv.cu",
           "moe_weights_file.cu", "moe_ep.cu", "moe_subspace.cu", "moe_dense.cu"]
OBJDIR = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + \
        [os.path.join(ROOT, "include", "moe_b200.h")]
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    # one nvcc per translation unit, in parallel, then one link
    os.makedirs(OBJDIR, exist_ok=True)
    procs, objs = [], []
    for src in sources():
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [NVCC, *ARCH, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-c", "-o", obj, src]
        procs.append((src, subprocess.Popen(cmd)))
    failed = [src for src, p in procs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, f"nvcc {failed}")
    subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-lcuda"], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    print(LIB)
