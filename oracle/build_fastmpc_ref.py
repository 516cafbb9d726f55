"""TEST INFRASTRUCTURE ONLY -- builds oracle/_ref/libfastmpc_ref.so: the
reference FastMPC extension's CUDA kernels, compiled from the reference's own
sources where they lie (differentialMPCPerformance/cpp, read in place, never
copied) with the CUDA flags its builder gives them (drone_ilqr.py: -O3
--use_fast_math, and the DRONE_ILQR_USE_* defines of the CUDA build, which
also leave out the file's standalone torch bindings), plus the extern "C" shim
in oracle/fastmpc_ref/shim.cu.

    python oracle/build_fastmpc_ref.py <reference root>

Runs only where the reference tree exists (the build container); the built
library travels with the repository to the GPU machine, where the parity
tests load it. Exits 0 with a message when the reference is absent.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libfastmpc_ref.so")
SOURCES = ("drone_kernels.cu", "forward_pass_kernel.cu", "backward_pass_kernel.cu", "pnqp_kernel.cu")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math", "-std=c++17",
         "-Xcompiler", "-fPIC", "-DDRONE_ILQR_USE_FUSED_BACKWARD", "-DDRONE_ILQR_USE_FUSED_FORWARD",
         "-DDRONE_ILQR_USE_PNQP", "-DDRONE_ILQR_USE_CUDA_KERNELS"]


def build(reference_root: str) -> str | None:
    cpp = os.path.join(reference_root, "differentialMPCPerformance", "cpp")
    if not all(os.path.exists(os.path.join(cpp, s)) for s in SOURCES):
        print(f"reference FastMPC sources not found under {cpp}; oracle/_ref not built")
        return None
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = [os.path.join(HERE, "fastmpc_ref", "shim.cu")] + [os.path.join(cpp, s) for s in SOURCES]
    newest = max(os.path.getmtime(s) for s in srcs + [os.path.abspath(__file__)])
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    cmd = [os.environ.get("NVCC", "nvcc"), *FLAGS, "-I", cpp, "-shared", "-o", OUT, *srcs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return OUT


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/build_fastmpc_ref.py <reference root>")
    print(build(sys.argv[1]))
