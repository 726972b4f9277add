"""Builds breadv2_b200/libbread_b200.so from csrc/*.cu for sm_100a (in-tree).

    python -m breadv2_b200.build [-v] [--force]

Every translation unit is compiled with relocatable device code (the device
error word is shared across units) and linked by nvcc into one shared library
exporting the C ABI of include/bread_b200.h.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbread_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", "-Wno-deprecated-gpu-targets"]

SOURCES = ["errors.cu", "gemv.cu", "gguf.cu", "glue.cu", "moe.cu", "moe_h1.cu", "moe_h2.cu", "moe_h4.cu", "moe_h8.cu",
           "moe_h16.cu", "noalloc.cu", "stack.cu", "synth.cu"]
HEADERS = ["common.cuh", "ptx.cuh", "qdot.cuh", "moe.cuh", "moe_kernel.cuh"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout + r.stderr, flush=True)


def build(verbose: bool = False, force: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "bread_b200.h")]
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or ptxas_v or _stale(o, [s, *hdrs, __file__]):
            extra = ["-Xptxas", "-v"] if ptxas_v else []
            jobs.append([NVCC, *ARCH, *FLAGS, *extra, "-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=min(12, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda c: _run(c, verbose or ptxas_v), jobs))
    if force or jobs or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB, "-lcudart"], verbose)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / spill / smem usage per kernel")
    a = ap.parse_args(argv)
    print(build(a.verbose, a.force, a.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
