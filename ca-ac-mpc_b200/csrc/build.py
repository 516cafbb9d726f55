"""Build libilqr_b200.so (the C-ABI solver library) in-tree for sm_100a.

    python ca-ac-mpc_b200/csrc/build.py [--verbose]

Compiles every .cu file in this directory with nvcc for sm_100a
(-gencode arch=compute_100a,code=sm_100a, -lineinfo, -fmad=false so the model
arithmetic rounds like the reference's elementwise torch ops; FILE_FLAGS adds
per-file options) and links them
into ca-ac-mpc_b200/libilqr_b200.so. Objects are rebuilt only when a source or
header is newer than the object (make-style), in parallel.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
OBJ_DIR = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(PKG, "libilqr_b200.so")
PROBE_LIB = os.path.join(PKG, "libilqr_probe.so")
PROBE_SRC = os.path.join(HERE, "probe", "fma_probe.cu")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-O2",
         "-I", os.path.join(ROOT, "include"), "-I", HERE]
# Per-file additions. The FastMPC numerics kernels restate a build compiled
# with --use_fast_math, whose divisions are the approximate (2-ulp) kind; they
# use that division too (at B = 16384 the solve takes 5.4 ms instead of 8.5 ms
# with IEEE division, inside the same parity bars).
FILE_FLAGS = {"ilqr_fastmpc.cu": ["-prec-div=false"]}


def _newer(src_files, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_files)


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    headers = sorted(glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(HERE, "*.h"))
                     + glob.glob(os.path.join(ROOT, "include", "*.h")))
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(OBJ_DIR, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        if _newer([src, os.path.abspath(__file__)] + headers, obj):
            cmd = [NVCC, *ARCH, *FLAGS, *FILE_FLAGS.get(os.path.basename(src), []), "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = False
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for cmd, r in ex.map(run, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed = True
                sys.stderr.write(" ".join(cmd) + "\n" + out + "\n")
            elif verbose and out:
                print(out)
    if failed:
        raise RuntimeError("nvcc failed")
    if jobs or _newer(objs, LIB):
        link = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    # FP32 FMA throughput probe used by the benchmark's roofline (separate
    # library: measurement only).
    if _newer([PROBE_SRC], PROBE_LIB):
        cmd = [NVCC, *ARCH, "-O3", "-Xcompiler", "-fPIC", "-shared", PROBE_SRC, "-o", PROBE_LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("probe build failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose))
