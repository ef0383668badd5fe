#!/usr/bin/env python
"""Build libatflash_b200.so (sm_100a) in-tree with nvcc.

    python atflash-kernel_b200/build.py [--verbose-ptxas]

The library is written to atflash-kernel_b200/atflash/_lib/ so that it travels
with the source tree; nothing is installed.
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "atflash", "_lib")
LIB = os.path.join(OUT_DIR, "libatflash_b200.so")
SOURCES = ["api.cu", "prefill_sm100.cu", "decode.cu", "decode_noalloc.cu", "exchange.cu", "rope.cu", "append.cu", "selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose_ptxas=False, force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(ROOT, "include", "atflash_b200.h"))
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= t for d in deps):
            return LIB
    cmd = [nvcc_path(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
           "-shared", "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp", *srcs]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
    sys.exit(0)
