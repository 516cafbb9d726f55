"""Generate golden vectors by running the reference DiffMPC solver itself.

Run in the build container, where the reference source tree is available:

    python tests/golden/make_golden.py --ref <reference root>

It imports the reference's DifferentialMPC package and DroneDx model from
their source tree (a stand-in module replaces matplotlib, which drone.py
imports only for plotting), runs fwd+bwd exactly as the policy's DiffMPC
backend does (DroneDxDiffMPCWrapper semantics, GradMethod.ANALYTIC,
detach_unconverged=False; acmpc_public-master/training_modules/
mlp_mpc_policy_diffmpc.py:34-43,114-162,261-280), and writes compressed
.npz fixtures next to this script.

The line search is instrumented (candidate costs and trajectories are
recorded per iteration) so that the reference's decision trace can be
reconstructed exactly. The script checks that the returned X, U are
bit-identical to the candidate accepted at each element's last improving
iteration, and reports how far a rejected element's recomputed candidate
costs drift between iterations (torch's CPU reductions are not bit-stable
across iterations) and how often that drift lets it improve again.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "ca-ac-mpc_b200"))
import ilqr_workload as wl  # noqa: E402

NOT_RUN = -128


def import_reference(ref_root):
    mpl = types.ModuleType("matplotlib")
    mpl.use = lambda *a, **k: None
    plt = types.ModuleType("matplotlib.pyplot")
    plt.style = types.SimpleNamespace(use=lambda *a, **k: None)
    mpl.pyplot = plt
    sys.modules.setdefault("matplotlib", mpl)
    sys.modules.setdefault("matplotlib.pyplot", plt)
    sys.path.insert(0, os.path.join(ref_root, "acmpc_public-master", "diff_mpc_drones"))
    sys.path.insert(0, os.path.join(ref_root, "acmpc_public-master", "mpc.pytorch"))
    sys.path.insert(0, ref_root)
    import drone  # noqa: F401
    import DifferentialMPC  # noqa: F401
    import DifferentialMPC.controller as ctl
    assert not ctl._HAS_SCAN, "reference must take its python-loop Riccati branch"
    return drone, DifferentialMPC


def import_policy_cost_builder(ref_root):
    """The policy's own cost construction, _build_cost_tensors
    (training_modules/mlp_mpc_policy_diffmpc.py:194-247). The module imports
    gym.spaces only for its class definitions: a stub stands in for it."""
    gym = types.ModuleType("gym")
    gym.spaces = types.ModuleType("gym.spaces")
    gym.spaces.Space = gym.spaces.Box = type("Space", (), {})
    sys.modules.setdefault("gym", gym)
    sys.modules.setdefault("gym.spaces", gym.spaces)
    sys.path.insert(0, os.path.join(ref_root, "acmpc_public-master", "training_modules"))
    import mlp_mpc_policy_diffmpc as pol
    return pol.CustomNetworkDiffMPC._build_cost_tensors


def run_reference(drone, DM, inp, T, max_iter, alphas, dt, bounds, gX, gU,
                  extra=None, reg=1e-6, model=None, dtype=None):
    """Run the reference DiffMPC fwd+bwd and record its decisions. `model`
    None is the reference's DroneDx with its analytic Jacobian; otherwise a
    dict(nx, f_dyn, u_min, u_max) run through GradMethod.AUTO_DIFF
    (controller.py:607-615), the controller's model-generic path. `dtype`
    (a torch dtype) runs the reference in that precision instead of float32."""
    import torch
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    B = inp["x0"].shape[0]
    if model is None:
        nx = 10
        dx = drone.DroneDx(device="cpu")
        dx.dt = dt
        f_dyn = lambda x, u, _dt: dx(x, u)
        f_jac = lambda x, u, _dt: dx.grad_input(x, u)
        gm = DM.GradMethod.ANALYTIC
        lo, hi = wl.U_MIN, wl.U_MAX
    else:
        nx, f_dyn, f_jac = model["nx"], model["f_dyn"], None
        gm = DM.GradMethod.AUTO_DIFF
        lo, hi = model["u_min"], model["u_max"]
    n = nx + 4
    cost = DM.GeneralQuadCost(nx=nx, nu=4, C=torch.zeros(1, T, n, n), c=torch.zeros(1, T, n),
                              C_final=torch.zeros(1, n, n), c_final=torch.zeros(1, n), device="cpu")
    u_min = torch.tensor(lo, dtype=dtype) if bounds else None
    u_max = torch.tensor(hi, dtype=dtype) if bounds else None
    ctrl = DM.DifferentiableMPCController(
        f_dyn=f_dyn, f_dyn_jac=f_jac, total_time=T * dt, step_size=dt, horizon=T,
        cost_module=cost, u_min=u_min, u_max=u_max, reg_eps=reg,
        grad_method=gm, max_iter=max_iter, exit_unconverged=False,
        detach_unconverged=False, device="cpu", verbose=0, use_vmap_line_search=False,
        alphas=tuple(alphas))
    t = lambda a: a if isinstance(a, torch.Tensor) else torch.tensor(a, dtype=dtype).clone().requires_grad_(True)
    x0, C, c = t(inp["x0"]), t(inp["C"]), t(inp["c"])  # C, c may come from a construction graph
    ex = extra or {}
    C_f = t(ex.get("C_final", np.zeros((B, n, n), np.float32)))
    c_f = t(ex.get("c_final", np.zeros((B, n), np.float32)))
    x_ref = t(ex.get("x_ref", np.zeros((B, T + 1, nx), np.float32)))
    u_ref = t(ex.get("u_ref", np.zeros((B, T, 4), np.float32)))
    cost.C, cost.c, cost.C_final, cost.c_final = C, c, C_f, c_f
    cost.set_reference(x_ref, u_ref)

    rec_costs, rec_X, rec_U, rec_obj = [], [], [], []
    orig_eval = ctrl.evaluate_alphas_batch_optimized
    orig_obj = cost.objective

    def eval_hook(*a, **k):
        Xc, Uc, costs = orig_eval(*a, **k)
        rec_costs.append(costs.detach().clone())
        rec_X.append(Xc.detach().clone())
        rec_U.append(Uc.detach().clone())
        return Xc, Uc, costs

    def obj_hook(*a, **k):
        out = orig_obj(*a, **k)
        rec_obj.append(out.detach().clone())
        return out

    ctrl.evaluate_alphas_batch_optimized = eval_hook
    cost.objective = obj_hook
    X, U = ctrl(x0, U_init=torch.tensor(inp["U_init"], dtype=dtype))
    converged = bool(ctrl.converged)
    tight = ctrl.tight_mask_last.detach().numpy().copy()
    L = (X * torch.tensor(gX, dtype=dtype)).sum() + (U * torch.tensor(gU, dtype=dtype)).sum()
    L.backward()

    # Reconstruct the decision trace exactly as solve_step decides. A rejected
    # element keeps X, U and its best cost; the reference recomputes its
    # candidates every later iteration and torch's CPU reductions are not
    # bit-stable across iterations, so a rejected element can occasionally
    # "re-improve" by a rounding-level margin. The trace records what the
    # reference actually did; drift and re-improvements are reported.
    best = rec_obj[0].clone()
    trace = np.full((B, max_iter), NOT_RUN, dtype=np.int8)
    last_acc, last_rej_costs = {}, {}
    drift, reimproved = 0.0, 0
    for i, costs in enumerate(rec_costs):
        j = torch.argmin(costs, dim=1)
        new = costs[torch.arange(B), j]
        improved = new < best
        for b in range(B):
            if b in last_rej_costs:
                old = last_rej_costs[b].double().min()
                d = abs(float(new[b]) - float(old)) / max(1.0, abs(float(old)))
                drift = max(drift, d)
            if bool(improved[b]):
                trace[b, i] = int(j[b])
                last_acc[b] = (i, int(j[b]))
                if b in last_rej_costs:
                    reimproved += 1
                    del last_rej_costs[b]
            else:
                trace[b, i] = -(int(j[b]) + 1)
                last_rej_costs[b] = costs[b].clone()
        best = torch.where(improved, new, best)
    for b in range(B):
        if b in last_acc:
            i, j = last_acc[b]
            assert torch.equal(X[b].detach(), rec_X[i][b, j]), "X is not the accepted candidate"
            assert torch.equal(U[b].detach(), rec_U[i][b, j]), "U is not the accepted candidate"
    g = lambda v: v.grad.detach().numpy().copy() if v.grad is not None else np.zeros(tuple(v.shape), np.float32)
    costs_all = torch.stack(rec_costs).numpy() if rec_costs else np.zeros((0, B, len(alphas)), np.float32)
    return dict(costs=costs_all, obj0=rec_obj[0].numpy().copy(),
                refreeze_drift=np.array(drift), reimproved=np.array(reimproved), X=X.detach().numpy().copy(), U=U.detach().numpy().copy(), trace=trace,
                best_cost=best.numpy().copy(), converged=np.array(converged),
                tight=tight, n_iter_run=np.array(len(rec_costs)),
                grad_x0=g(x0), grad_C=g(C), grad_c=g(c), grad_C_final=g(C_f),
                grad_c_final=g(c_f), grad_xref=g(x_ref), grad_uref=g(u_ref))


CASES = {
    # name: (config or None, B, T, max_iter, alphas, bounds, extra-kind)
    "cfg1_b16_t5": ("latency_b16_t5", 16, None, None, None, True, None),
    "cfg2_b32_t10": ("b1024_t10", 32, None, None, None, True, None),
    "cfg3_b16_t20": ("rollout_b16384_t20", 16, None, None, None, True, None),
    "cfg5_b64_t50": ("stress_b65536_t50", 64, None, None, None, True, None),
    "dense_b8_t6": (None, 8, 6, 6, (1.0, 0.8, 0.5, 0.2, 0.1), True, "dense"),
    "asym_b8_t4": (None, 8, 4, 5, (1.0, 0.8, 0.5, 0.2, 0.1), True, "asym"),
    "nobox_b8_t5": (None, 8, 5, 6, (1.0, 0.8, 0.5, 0.2, 0.1), False, None),
    "b1_t1": (None, 1, 1, 3, (1.0, 0.8, 0.5, 0.2, 0.1), True, None),
    "indef_b8_t4": (None, 8, 4, 3, (1.0, 0.8, 0.5, 0.2, 0.1), True, "indef"),
}


def make_case(drone, DM, name):
    cfg_name, B, T, max_iter, alphas, bounds, kind = CASES[name]
    if cfg_name is not None:
        cfg, inp = wl.config_inputs(cfg_name, B=B, seed=0)
        T, max_iter, alphas = cfg["T"], cfg["max_iter"], cfg["alphas"]
    else:
        inp = wl.make_inputs(B, T, seed=3)
    extra = None
    if kind == "indef":
        # A negative control weight on some elements makes Q_uu indefinite, so
        # the reference's Cholesky fails and its SVD inverse is used.
        for b in range(0, B, 2):
            inp["C"][b, :, 11, 11] = -0.05
    if kind in ("dense", "asym"):
        extra = wl.make_dense_costs(B, T, seed=11, asymmetric=(kind == "asym"))
        inp["C"], inp["c"] = extra.pop("C"), extra.pop("c")
    gX, gU = wl.make_backward_seeds(B, T, seed=1)
    out = run_reference(drone, DM, inp, T, max_iter, alphas, wl.DT, bounds, gX, gU, extra)
    arrays = dict(inp)
    if extra:
        arrays.update(extra)
    arrays.update(gX=gX, gU=gU, dt=np.array(wl.DT), max_iter=np.array(max_iter),
                  alphas=np.array(alphas, dtype=np.float32), bounds=np.array(bounds),
                  reg=np.array(1e-6), converge_tol=np.array(1e-6))
    arrays.update({"ref_" + k: v for k, v in out.items()})
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    tf = out["tight"].mean() if bounds else 0.0
    print(f"{name}: B={B} T={T} iters={max_iter} run={int(out['n_iter_run'])} "
          f"converged={bool(out['converged'])} tight={tf:.3f} refreeze_drift={float(out['refreeze_drift']):.1e} reimproved={int(out['reimproved'])} -> {os.path.getsize(path)/1e3:.0f} kB")


def make_sigmoid_case(drone, DM, build, name="sigmoid_b16_t10", B=16, T=10, max_iter=5):
    """Costs from the policy's sigmoid output: the reference's construction
    feeds DiffMPC, and the gradient flows back to the sigmoid output."""
    import torch
    rng = np.random.default_rng(21)
    sc = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.5, (B, 28 * T))))).astype(np.float32)
    inp = wl.make_inputs(B, T, seed=4)
    dx = types.SimpleNamespace(n_state=10, n_ctrl=4, mass=0.752)
    fake = types.SimpleNamespace(T=T, dx=dx, mpc_device=torch.device("cpu"))
    sct = torch.tensor(sc).requires_grad_(True)
    C, c, Cf, cf = build(fake, sct)
    inp_t = dict(x0=inp["x0"], U_init=inp["U_init"], C=C, c=c)
    gX, gU = wl.make_backward_seeds(B, T, seed=1)
    alphas = (1.0, 0.8, 0.5, 0.2, 0.1)
    out = run_reference(drone, DM, inp_t, T, max_iter, alphas, wl.DT, True, gX, gU)
    arrays = dict(x0=inp["x0"], U_init=inp["U_init"], sigmoid_cost=sc,
                  C=C.detach().numpy().copy(), c=c.detach().numpy().copy())
    arrays.update(gX=gX, gU=gU, dt=np.array(wl.DT), max_iter=np.array(max_iter),
                  alphas=np.array(alphas, dtype=np.float32), bounds=np.array(True),
                  reg=np.array(1e-6), converge_tol=np.array(1e-6),
                  cost_eps=np.array(0.1), range_q=np.array(100000.0), range_p=np.array(100000.0),
                  range_pt=np.array(100000.0 * 0.752 * 9.806))
    arrays.update({"ref_" + k: v for k, v in out.items() if k not in ("grad_C", "grad_c")})
    arrays["ref_grad_sigmoid_cost"] = sct.grad.detach().numpy().copy()
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"{name}: B={B} T={T} iters={max_iter} run={int(out['n_iter_run'])} "
          f"tight={out['tight'].mean():.3f} -> {os.path.getsize(path)/1e3:.0f} kB")


def make_dynamics(drone):
    import torch
    rng = np.random.default_rng(5)
    n = 64
    x = np.zeros((n, 10), np.float32)
    x[:, 0:3] = rng.normal(0, 2, (n, 3))
    q = rng.normal(size=(n, 4))
    x[:, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True) * rng.uniform(0.9, 1.1, (n, 1))
    x[:, 7:10] = rng.normal(0, 3, (n, 3))
    u = np.zeros((n, 4), np.float32)
    u[:, 0] = rng.uniform(0, 34, n)
    u[:, 1:4] = rng.uniform(-10, 10, (n, 3))
    u[:4, 1:4] = 0.0  # zero body rates exercise the normalize() eps branch
    dx = drone.DroneDx(device="cpu")
    dx.dt = wl.DT
    with torch.no_grad():
        xn = dx(torch.tensor(x), torch.tensor(u)).numpy()
        A, Bm = dx.grad_input(torch.tensor(x), torch.tensor(u))
    path = os.path.join(HERE, "dynamics_n64.npz")
    np.savez_compressed(path, x=x, u=u, dt=np.array(wl.DT), x_next=xn, A=A.numpy(), B=Bm.numpy())
    print(f"dynamics_n64 -> {os.path.getsize(path)/1e3:.0f} kB")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference source tree")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    drone, DM = import_reference(args.ref)
    if not args.only:
        make_dynamics(drone)
    for name in CASES:
        if args.only and name not in args.only:
            continue
        make_case(drone, DM, name)
    if not args.only or "sigmoid_b16_t10" in args.only:
        make_sigmoid_case(drone, DM, import_policy_cost_builder(args.ref))


if __name__ == "__main__":
    main()
