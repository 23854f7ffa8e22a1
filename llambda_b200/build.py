"""Builds libllambda_cuda.so in-tree with nvcc for sm_100a (B200).

Usage: python -m llambda_b200.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libllambda_cuda.so")

CU_SOURCES = ["gemv.cu", "moe.cu", "prefill.cu", "gguf.cu", "capi.cu"]
C_SOURCES = ["sha256.c"]
HEADERS = ["common.cuh", "engine.cuh", "kernels.h", "synth.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_input() -> float:
    paths = [os.path.join(CSRC, f) for f in CU_SOURCES + C_SOURCES + HEADERS]
    paths.append(os.path.join(ROOT, "include", "llambda_cuda.h"))
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def needs_build() -> bool:
    return not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest_input()


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    jobs = []
    for src in CU_SOURCES:
        obj = os.path.join(BUILD, src + ".o")
        jobs.append([nv, *ARCH, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj])
    for src in C_SOURCES:
        obj = os.path.join(BUILD, src + ".o")
        jobs.append(["gcc", "-O3", "-fPIC", "-fvisibility=hidden", "-c", os.path.join(CSRC, src),
                     "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out.strip():
                print(out)
    vscript = os.path.join(BUILD, "exports.map")
    with open(vscript, "w") as f:
        f.write("{ global: llambda_cuda_*; local: *; };\n")
    objs = [os.path.join(BUILD, s + ".o") for s in CU_SOURCES + C_SOURCES]
    tmp = LIB + ".tmp"
    _run([nv, *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static",
          "-Xlinker", "--version-script=" + vscript, "-Xlinker", "-z,defs", "-lrt", "-ldl",
          "-lpthread"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
