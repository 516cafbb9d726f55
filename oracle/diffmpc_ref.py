"""TEST AND BASELINE INFRASTRUCTURE ONLY -- runs the reference DiffMPC solver
itself (the sources oracle/stage_diffmpc_ref.py copied into
oracle/_ref/diffmpc/) on the host CPU, as the policy's "diffmpc" backend
calls it: DroneDx with its analytic Jacobian (DroneDxDiffMPCWrapper,
acmpc_public-master/training_modules/mlp_mpc_policy_diffmpc.py:34-43),
GeneralQuadCost with the chunk's C, c and zero terminal cost and references
(:261-280), DifferentiableMPCController with GradMethod.ANALYTIC,
detach_unconverged=False and the control box (:114-162), then the implicit
backward of a scalar loss through ILQRSolve (DifferentialMPC/controller.py:
31-133). Only the benchmark's CPU-baseline leg and its reference arm use it;
the product never imports anything under oracle/.
"""

from __future__ import annotations

import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
STAGED = os.path.join(HERE, "_ref", "diffmpc")


def available() -> bool:
    return os.path.isfile(os.path.join(STAGED, "DifferentialMPC", "controller.py")) and \
        os.path.isfile(os.path.join(STAGED, "drone.py"))


def _import():
    """Import the staged reference (a stand-in replaces matplotlib, which
    drone.py imports only for plotting)."""
    mpl = types.ModuleType("matplotlib")
    mpl.use = lambda *a, **k: None
    plt = types.ModuleType("matplotlib.pyplot")
    plt.style = types.SimpleNamespace(use=lambda *a, **k: None)
    mpl.pyplot = plt
    sys.modules.setdefault("matplotlib", mpl)
    sys.modules.setdefault("matplotlib.pyplot", plt)
    if STAGED not in sys.path:
        sys.path.insert(0, STAGED)
    import drone
    import DifferentialMPC as DM
    return drone, DM


def solve_fwd_bwd(inp, T, max_iter, alphas, dt, u_min, u_max, gX, gU, reg=1e-6):
    """One fwd+bwd solve of the batch `inp` (numpy float32: x0, C, c, U_init)
    by the reference DiffMPC; returns X, U, dL/dx0 as numpy."""
    import torch
    drone, DM = _import()
    B = inp["x0"].shape[0]
    nx, nu = 10, 4
    n = nx + nu
    dx = drone.DroneDx(device="cpu")
    dx.dt = dt
    cost = DM.GeneralQuadCost(nx=nx, nu=nu, C=torch.zeros(1, T, n, n), c=torch.zeros(1, T, n),
                              C_final=torch.zeros(1, n, n), c_final=torch.zeros(1, n), device="cpu")
    ctrl = DM.DifferentiableMPCController(
        f_dyn=lambda x, u, _dt: dx(x, u), f_dyn_jac=lambda x, u, _dt: dx.grad_input(x, u),
        total_time=T * dt, step_size=dt, horizon=T, cost_module=cost,
        u_min=torch.tensor(u_min), u_max=torch.tensor(u_max), reg_eps=reg,
        grad_method=DM.GradMethod.ANALYTIC, max_iter=max_iter, exit_unconverged=False,
        detach_unconverged=False, device="cpu", verbose=0, alphas=tuple(alphas))
    x0 = torch.tensor(inp["x0"]).requires_grad_(True)
    C = torch.tensor(inp["C"]).requires_grad_(True)
    c = torch.tensor(inp["c"]).requires_grad_(True)
    cost.C, cost.c = C, c
    cost.C_final = torch.zeros(B, n, n)
    cost.c_final = torch.zeros(B, n)
    cost.set_reference(torch.zeros(B, T + 1, nx), torch.zeros(B, T, nu))
    X, U = ctrl(x0, U_init=torch.tensor(inp["U_init"]))
    ((X * torch.tensor(gX)).sum() + (U * torch.tensor(gU)).sum()).backward()
    return X.detach().numpy(), U.detach().numpy(), x0.grad.numpy()


def timed_rate(inp, T, max_iter, alphas, dt, u_min, u_max, gX, gU, threads, reps=1):
    """Element solves per second of solve_fwd_bwd on `threads` torch threads
    (best of `reps` runs after one warm-up run)."""
    import torch
    torch.set_num_threads(threads)
    solve_fwd_bwd(inp, T, max_iter, alphas, dt, u_min, u_max, gX, gU)
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        solve_fwd_bwd(inp, T, max_iter, alphas, dt, u_min, u_max, gX, gU)
        el = time.perf_counter() - t0
        best = el if best is None else min(best, el)
    return inp["x0"].shape[0] / best, best
