"""Generate the rotor13 golden vectors by running the reference DiffMPC on the
13-state rotor-thrust quadrotor.

The reference has no 13-state model (its solver and environment use the
10-state CTBR DroneDx). DiffMPC's controller is model-generic: given f_dyn
alone it linearises with GradMethod.AUTO_DIFF, jacrev under vmap
(DifferentialMPC/controller.py:607-615). This script writes the model below
as that f_dyn and runs the reference's own solver and implicit-diff backward
on it, exactly as make_golden.py does for DroneDx. The solver is therefore
pinned by the reference; the model is written here and is pinned by nothing
in the reference ("model unpinned by the reference"). The model is the one
oracle/rotor13_model.py restates in numpy (same expressions, same order).

Run in the build container (it imports the reference from its source tree):
    python tests/golden/make_rotor13_golden.py --ref <reference root>
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "ca-ac-mpc_b200"))

import ilqr_workload as wl  # noqa: E402
from make_golden import import_reference, run_reference  # noqa: E402

# float32 values of the model's derived constants (F_MAX / m, d F_MAX / J,
# KAPPA F_MAX / Jz, gyroscopic ratios, g), computed in float64 and rounded once.
ARM, JX, JY, JZ, KAPPA, F_MAX, MASS, G = 0.15, 2.5e-3, 2.5e-3, 4.5e-3, 0.016, 8.5, 0.75, 9.8066
_D = ARM / np.sqrt(2.0)
K32 = {k: float(np.float32(v)) for k, v in dict(
    FM=F_MAX / MASS, RX=_D * F_MAX / JX, RY=_D * F_MAX / JY, RZ=KAPPA * F_MAX / JZ,
    AX=(JY - JZ) / JX, AY=(JZ - JX) / JY, AZ=(JX - JY) / JZ, G=G).items()}


def rotor13_f_dyn(x, u, dt):
    """x + dt f(x, u) for x [..., 13], u [..., 4] (batched or single, as the
    controller's rollout and its vmap'd jacrev call it)."""
    import torch
    k = {n: torch.tensor(v, dtype=x.dtype) for n, v in K32.items()}
    half = torch.tensor(0.5, dtype=x.dtype)
    two = torch.tensor(2.0, dtype=x.dtype)
    qw, qx, qy, qz = x[..., 3], x[..., 4], x[..., 5], x[..., 6]
    wx, wy, wz = x[..., 10], x[..., 11], x[..., 12]
    u0, u1, u2, u3 = u[..., 0], u[..., 1], u[..., 2], u[..., 3]
    qd = [half * (-qx * wx - qy * wy - qz * wz),
          half * (qw * wx + qy * wz - qz * wy),
          half * (qw * wy - qx * wz + qz * wx),
          half * (qw * wz + qx * wy - qy * wx)]
    aT = k["FM"] * (((u0 + u1) + u2) + u3)
    r0 = two * (qw * qy + qx * qz)
    r1 = two * (qy * qz - qw * qx)
    r2 = ((qw * qw - qx * qx) - qy * qy) + qz * qz
    vd = [aT * r0, aT * r1, aT * r2 - k["G"]]
    wd = [k["RX"] * (((u0 - u1) - u2) + u3) + k["AX"] * (wy * wz),
          k["RY"] * (((u2 + u3) - u0) - u1) + k["AY"] * (wz * wx),
          k["RZ"] * (((u0 - u1) + u2) - u3) + k["AZ"] * (wx * wy)]
    xdot = torch.stack([x[..., 7], x[..., 8], x[..., 9]] + qd + vd + wd, dim=-1)
    return x + torch.tensor(dt, dtype=x.dtype) * xdot


MODEL = dict(nx=13, f_dyn=rotor13_f_dyn, u_min=wl.U_MIN13, u_max=wl.U_MAX13)

# The T=50 long-horizon configuration has no rotor13 case: on this model the
# reference DiffMPC itself fails there (from the hover linearisation its
# expanded V update loses definiteness about 25 steps from the horizon end,
# V grows past 1e10, and the SVD fallback raises on a non-finite Q_uu).
CASES = {
    # name: (config or None, B, T, max_iter, alphas, bounds, extra-kind)
    "r13_cfg1_b16_t5": ("latency_b16_t5", 16, None, None, None, True, None),
    "r13_cfg2_b32_t10": ("b1024_t10", 32, None, None, None, True, None),
    "r13_cfg3_b16_t20": ("rollout_b16384_t20", 16, None, None, None, True, None),
    "r13_dense_b8_t6": (None, 8, 6, 6, (1.0, 0.8, 0.5, 0.2, 0.1), True, "dense"),
    "r13_nobox_b8_t5": (None, 8, 5, 6, (1.0, 0.8, 0.5, 0.2, 0.1), False, None),
}


def dense_costs13(B, T, seed):
    """General SPD costs plus terminal cost and references for 17-wide tau."""
    rng = np.random.default_rng(seed)
    n = wl.N13
    Gm = rng.normal(size=(B, T, n, n)) * 0.3
    C = Gm @ np.swapaxes(Gm, -1, -2) / n
    C += np.eye(n) * np.exp(rng.uniform(np.log(1e-1), np.log(1e1), (B, T, n)))[..., None]
    c = rng.normal(0.0, 5.0, size=(B, T, n))
    Gf = rng.normal(size=(B, n, n)) * 0.3
    C_f = Gf @ np.swapaxes(Gf, -1, -2) / n
    c_f = rng.normal(0.0, 1.0, size=(B, n))
    x_ref = rng.normal(0.0, 0.1, size=(B, T + 1, wl.NX13))
    u_ref = rng.normal(0.0, 0.05, size=(B, T, wl.NU))
    f = lambda a: a.astype(np.float32)
    return dict(C=f(C), c=f(c), C_final=f(C_f), c_final=f(c_f), x_ref=f(x_ref), u_ref=f(u_ref))


def make_case(DM, name):
    cfg_name, B, T, max_iter, alphas, bounds, kind = CASES[name]
    if cfg_name is not None:
        cfg, inp = wl.rotor13_config_inputs(cfg_name, B=B, seed=0)
        T, max_iter, alphas = cfg["T"], cfg["max_iter"], cfg["alphas"]
    else:
        inp = wl.make_rotor13_inputs(B, T, seed=3)
    extra = None
    if kind == "dense":
        extra = dense_costs13(B, T, seed=11)
        inp["C"], inp["c"] = extra.pop("C"), extra.pop("c")
    gX, gU = wl.make_backward_seeds(B, T, seed=1, nx=wl.NX13)
    out = run_reference(None, DM, inp, T, max_iter, alphas, wl.DT, bounds, gX, gU,
                        dict(extra) if extra else None, model=MODEL)
    # The same problem through the reference in float64: on this model the
    # fp32 solve is strongly rounding-sensitive, and the fp64 run pins the
    # oracle's arithmetic independently of that.
    import torch
    out64 = run_reference(None, DM, inp, T, max_iter, alphas, wl.DT, bounds, gX, gU,
                          dict(extra) if extra else None, model=MODEL, dtype=torch.float64)
    arrays = dict(inp)
    if extra:
        arrays.update(extra)
    arrays.update(gX=gX, gU=gU, dt=np.array(wl.DT), max_iter=np.array(max_iter),
                  alphas=np.array(alphas, dtype=np.float32), bounds=np.array(bounds),
                  reg=np.array(1e-6), converge_tol=np.array(1e-6), model=np.array("rotor13"),
                  u_min=wl.U_MIN13, u_max=wl.U_MAX13)
    arrays.update({"ref_" + k: v for k, v in out.items()})
    arrays.update({"ref64_" + k: out64[k] for k in ("X", "U", "trace", "tight", "grad_x0", "grad_C", "grad_c",
                                                     "grad_C_final", "grad_c_final", "grad_xref", "grad_uref")})
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    tf = out["tight"].mean() if bounds else 0.0
    print(f"{name}: B={B} T={T} iters={max_iter} run={int(out['n_iter_run'])} "
          f"converged={bool(out['converged'])} tight={tf:.3f} "
          f"refreeze_drift={float(out['refreeze_drift']):.1e} reimproved={int(out['reimproved'])} "
          f"-> {os.path.getsize(path)/1e3:.0f} kB")


def make_dynamics():
    """f_dyn and its AUTO_DIFF Jacobian (jacrev under vmap, as the controller
    takes it) at 64 random states and controls."""
    import torch
    from torch.func import jacrev, vmap
    rng = np.random.default_rng(5)
    n = 64
    x = np.zeros((n, 13), np.float32)
    x[:, 0:3] = rng.normal(0, 2, (n, 3))
    q = rng.normal(size=(n, 4))
    x[:, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True) * rng.uniform(0.9, 1.1, (n, 1))
    x[:, 7:10] = rng.normal(0, 3, (n, 3))
    x[:, 10:13] = rng.normal(0, 4, (n, 3))
    u = rng.uniform(0, 1, (n, 4)).astype(np.float32)
    xt, ut = torch.tensor(x), torch.tensor(u)
    f = lambda a, b: rotor13_f_dyn(a, b, wl.DT)
    with torch.no_grad():
        xn = f(xt, ut).numpy()
    A = vmap(jacrev(f, argnums=0))(xt, ut).detach().numpy()
    Bm = vmap(jacrev(f, argnums=1))(xt, ut).detach().numpy()
    path = os.path.join(HERE, "r13_dynamics_n64.npz")
    np.savez_compressed(path, x=x, u=u, dt=np.array(wl.DT), x_next=xn, A=A, B=Bm)
    print(f"r13_dynamics_n64 -> {os.path.getsize(path)/1e3:.0f} kB")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference source tree")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    _, DM = import_reference(args.ref)
    if not args.only:
        make_dynamics()
    for name in CASES:
        if args.only and name not in args.only:
            continue
        make_case(DM, name)


if __name__ == "__main__":
    main()
