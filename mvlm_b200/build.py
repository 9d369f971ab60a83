"""Build libmgpu.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python -m mvlm_b200.build            # incremental
    python -m mvlm_b200.build --force    # rebuild everything

Objects go to mvlm_b200/_build/ (git-ignored); the library lands at mvlm_b200/libmgpu.so so
that it travels with the repository snapshot to the GPU host.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmgpu.so")
SOURCES = ["runtime.cu", "gemv.cu", "chain.cu", "gemm_tc.cu", "skinny.cu", "misc.cu", "peer.cu"]
HEADERS = ["common.cuh", "kernels.h", "qdot.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-ccbin", "g++"]


def _newer(src: str, dst: str) -> bool:
    return not os.path.exists(dst) or os.path.getmtime(src) > os.path.getmtime(dst)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = [os.path.join(CSRC, h) for h in HEADERS]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "mgpu_cuda.h"))
    objs, jobs = [], []
    relinked = force or not os.path.exists(LIB)
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        objs.append(obj)
        stale = force or _newer(src, obj) or any(_newer(d, obj) for d in deps)
        if not stale:
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd))
        jobs.append((s, cmd))
    # the translation units are independent: compile them side by side
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        results = list(pool.map(lambda j: (j[0], subprocess.run(j[1], capture_output=True, text=True)), jobs))
    for s, r in results:
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s}:\n{r.stdout}\n{r.stderr}")
        if verbose or ptxas_info:
            sys.stdout.write(r.stderr)
        relinked = True
    if relinked:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
