"""Golden vectors for the 4-dimensional box-constrained QP
(drone_pnqp4_batch, differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:1285-1316):
random positive-definite problems solved by the reference's specification,
mpc.pytorch's pnqp (acmpc_public-master/mpc.pytorch/mpc/pnqp.py:5-84), run
here on CPU in float64 with more iterations so that its x* is the converged
optimum (unique: H is positive definite). Writes pnqp4_n256.npz.

Usage: python tests/golden/make_pnqp_golden.py --ref <reference root>
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference source tree")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "acmpc_public-master", "mpc.pytorch"))
    import torch
    from mpc.pnqp import pnqp

    rng = np.random.default_rng(13)
    n = 256
    G = rng.normal(size=(n, 4, 4))
    H = G @ np.swapaxes(G, 1, 2) + np.eye(4) * rng.uniform(0.05, 2.0, (n, 1, 1))
    q = rng.normal(0.0, 3.0, (n, 4))
    lo = -rng.uniform(0.1, 2.0, (n, 4))
    hi = rng.uniform(0.1, 2.0, (n, 4))
    lo[:32] = -1e3  # some problems with no active bound
    hi[:32] = 1e3
    f32 = lambda a: a.astype(np.float32)
    H, q, lo, hi = f32(H), f32(q), f32(lo), f32(hi)
    x, _, If, _ = pnqp(torch.tensor(H, dtype=torch.float64), torch.tensor(q, dtype=torch.float64),
                       torch.tensor(lo, dtype=torch.float64), torch.tensor(hi, dtype=torch.float64),
                       n_iter=200)
    opt = np.stack([exact_box_qp(H[b].astype(np.float64), q[b].astype(np.float64), lo[b].astype(np.float64),
                                 hi[b].astype(np.float64)) for b in range(n)])
    np.savez_compressed(os.path.join(HERE, "pnqp4_n256.npz"), H=H, q=q, lower=lo, upper=hi,
                        ref_x=x.numpy(), ref_free=If.numpy(), opt_x=opt)
    reached = np.abs(x.numpy() - opt).max(axis=1) <= 1e-6
    print("pnqp4_n256: active fraction", float(1 - If.numpy().mean()),
          "| mpc.pytorch pnqp reached the exact optimum on", int(reached.sum()), "of", n)


def exact_box_qp(H, q, lo, hi):
    """Exact minimiser of 1/2 x^T H x + q^T x on a 4-d box (H positive
    definite): every pattern of free / at-lower / at-upper coordinates, the
    free block solved in float64, the feasible candidate of least objective."""
    import itertools
    best, best_obj = None, np.inf
    for pat in itertools.product((0, 1, 2), repeat=4):
        x = np.zeros(4)
        fixed = [i for i in range(4) if pat[i] != 0]
        free = [i for i in range(4) if pat[i] == 0]
        for i in fixed:
            x[i] = lo[i] if pat[i] == 1 else hi[i]
        if free:
            rhs = -q[free] - H[np.ix_(free, fixed)] @ x[fixed] if fixed else -q[free]
            x[free] = np.linalg.solve(H[np.ix_(free, free)], rhs)
        if np.any(x < lo - 1e-12) or np.any(x > hi + 1e-12):
            continue
        o = 0.5 * x @ H @ x + q @ x
        if o < best_obj:
            best, best_obj = x, o
    return best


if __name__ == "__main__":
    main()
