"""Builds libcuda_fletcher.so (sm_100a) in-tree with nvcc.

    python longbow-fletcher_b200/build.py [--force]

Objects go to longbow-fletcher_b200/_build/, the library next to this file.  The CUDA runtime
is linked statically so the library only needs the driver at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcuda_fletcher.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DFLETCHER_BUILD"]
SOURCES = ["context.cu", "ops.cu", "gemm_simt.cu", "gemm_tc.cu", "attention.cu", "model.cu", "abi_ops.cu",
           "noalloc.cu", "attention_tc.cu", "probe.cu", "runtime.cu"]


def _deps():
    out = []
    for d in (CSRC, os.path.join(os.path.dirname(HERE), "include")):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h")):
                out.append(os.path.join(d, f))
    return out


def _stale(target, inputs):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def _compile(src, verbose=False):
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    todo = [s for s in srcs if force or _stale(os.path.join(BUILD, os.path.basename(s).replace(".cu", ".o")), [s, *deps])]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
            if verbose and log:
                print(log, file=sys.stderr)
    objs = [os.path.join(BUILD, os.path.basename(s).replace(".cu", ".o")) for s in srcs]
    if force or todo or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
