"""Generate the FastMPC golden fixtures (fm_ref_*.npz) by running the
reference FastMPC extension's CUDA build: its own kernels, compiled from the
reference sources into oracle/_ref/libfastmpc_ref.so by
oracle/build_fastmpc_ref.py, driven by oracle/fastmpc_ref_cuda.py (the restated host
loop of drone_ilqr_solve, differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:
664-1064, and of the operator's CUDA backward, differentialMPCPerformance/
mpc_compat.py:217-258). Needs a GPU.

Each fixture holds the inputs, the reference's free-running decision trace,
the iterations the batch ran, its X, U and tight mask, the candidate costs of
every iteration, and the gradients of x0, C, c for seeded dL/dX, dL/dU.

    python tests/golden/make_fastmpc_golden.py [out_dir]
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "ca-ac-mpc_b200")]

from oracle import fastmpc_ref_cuda as ref  # noqa: E402
import ilqr_workload as wl  # noqa: E402

LO = np.array([0.0, -10.0, -10.0, -4.0], np.float32)
HI = np.array([34.0, 10.0, 10.0, 4.0], np.float32)


def cases():
    """(name, inputs, boxed, max_iter): the policy's box and dt = 0.05, zero
    terminal cost and references, as the FastMPC operator passes them."""
    d = wl.make_inputs(8, 6, seed=3)
    dense = wl.make_dense_costs(8, 6, seed=4)
    return [
        ("fm_ref_cfg1_b16_t5", wl.make_inputs(16, 5, seed=0), True, 10),
        ("fm_ref_cfg2_b24_t10", wl.make_inputs(24, 10, seed=1), True, 10),
        ("fm_ref_cfg3_b12_t20", wl.make_inputs(12, 20, seed=2), True, 5),
        ("fm_ref_dense_b8_t6", dict(d, C=dense["C"], c=dense["c"]), True, 6),
        ("fm_ref_nobox_b8_t5", wl.make_inputs(8, 5, seed=5), False, 5),
        ("fm_ref_ragged_b13_t7", wl.make_inputs(13, 7, seed=6, r=15.0), True, 9),
        ("fm_ref_cfg5_b8_t50", wl.make_inputs(8, 50, seed=7, r=15.0), True, 8),
    ]


def main(out_dir):
    if not torch.cuda.is_available() or not ref.available():
        raise SystemExit("needs a GPU and oracle/_ref/libfastmpc_ref.so")
    os.makedirs(out_dir, exist_ok=True)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a)).to("cuda", torch.float32)
    for name, d, boxed, iters in cases():
        B, T = d["U_init"].shape[:2]
        lo, hi = (t(LO), t(HI)) if boxed else (None, None)
        r = ref.solve(t(d["x0"]), t(d["U_init"]), t(d["C"]), t(d["c"]), lo, hi, dt=0.05, max_iter=iters)
        gX, gU = wl.make_backward_seeds(B, T)
        g = ref.backward(r, t(gX), t(gU))
        n = lambda x: x.detach().cpu().numpy()
        np.savez_compressed(
            os.path.join(out_dir, name + ".npz"),
            x0=d["x0"].astype(np.float32), U_init=d["U_init"].astype(np.float32),
            C=d["C"].astype(np.float32), c=d["c"].astype(np.float32), boxed=np.bool_(boxed),
            u_min=LO, u_max=HI, dt=np.float32(0.05), max_iter=np.int64(iters), gX=gX.astype(np.float32),
            gU=gU.astype(np.float32), ref_X=n(r["X"]), ref_U=n(r["U"]), ref_tight=n(r["tight"]),
            ref_trace=n(r["trace"]), ref_iters=np.int64(r["iters"]), ref_converged=np.bool_(r["converged"]),
            ref_costs=n(r["costs"]), ref_best_before=n(r["best_before"]), ref_x0=n(g["x0"]), ref_C=n(g["C"]),
            ref_c=n(g["c"]))
        print(name, "iters", r["iters"], "converged", r["converged"])


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
