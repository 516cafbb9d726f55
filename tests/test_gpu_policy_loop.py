"""The policy actor's MPC step as one batched call (policy_mpc.PolicyMPC)
against a restatement of the reference's chunked loop
(CustomNetworkDiffMPC.forward_actor, training_modules/mlp_mpc_policy_diffmpc.py:300-434)
run on the same solver with dense costs built chunk by chunk."""

import numpy as np
import pytest
import torch

import mpc_compat
import oracle as O
import policy_mpc
import ilqr_workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
T, DT, MASS = 10, 0.05, 0.752


def _reference_loop(sc, states, u_prev, chunk, lqr_iter, eps, numerics=None):
    """forward_actor's loop: per chunk, dense C, c from the sigmoid output,
    U_init from the warm start (or hover), FastMPC solve; then the warm start
    update and the action normalisation."""
    B = states.shape[0]
    lo = torch.tensor([0.0, -10.0, -10.0, -4.0], device=DEV)
    hi = torch.tensor([34.0, 10.0, 10.0, 4.0], device=DEV)
    mpc = mpc_compat.FastMPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                             u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=lqr_iter, eps=eps,
                             numerics=numerics)
    dx = type("Dx", (), {"dt": DT})()
    nom_u = torch.zeros(B, T, 4, device=DEV)
    naninf = 0
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        C, c = O.sigmoid_costs(sc[s:e].cpu().numpy(), T)
        U_init = u_prev[s:e].unsqueeze(1).expand(-1, T, -1).clone()
        mpc.u_init = U_init.permute(1, 0, 2).contiguous()
        cost = mpc_compat.QuadCost(torch.from_numpy(C).to(DEV).permute(1, 0, 2, 3).contiguous(),
                                   torch.from_numpy(c).to(DEV).permute(1, 0, 2).contiguous())
        with torch.no_grad():
            _, U_tbn, _ = mpc(states[s:e, :10], cost, dx)
        U = U_tbn.permute(1, 0, 2)
        nom_u[s:e] = U
        naninf += int((~torch.isfinite(U)).any().item())
    thrust = nom_u[:, 0, 0] / MASS
    force_std = max(1e-6, 8.5 * 4 / MASS - 9.8066)
    act = torch.cat((((thrust - 9.8066) / force_std).unsqueeze(1),
                     nom_u[:, 0, 1:4] / torch.tensor([10.0, 10.0, 4.0], device=DEV)), dim=1)
    return act, nom_u[:, 0, :].clone(), naninf


def test_actor_matches_chunked_reference_loop_with_warm_start():
    B = 37
    rng = np.random.default_rng(4)
    inp = wl.make_inputs(B, T, seed=6)
    states = torch.from_numpy(inp["x0"]).to(DEV)
    pm = policy_mpc.PolicyMPC(T, DT, lqr_iter=3, eps=0.1, chunk=8, device=DEV)
    u_prev = torch.zeros(B, 4, device=DEV)
    u_prev[:, 0] = MASS * 9.8066
    for call in range(2):  # the second call starts from the first call's warm start
        sc = torch.from_numpy((1 / (1 + np.exp(-rng.normal(0, 1.5, (B, 28 * T))))).astype(np.float32)).to(DEV)
        with torch.no_grad():
            act = pm.actor(sc, states)
        ref_act, ref_u_prev, ref_naninf = _reference_loop(sc, states, u_prev, 8, 3, 0.1)
        assert torch.equal(act, ref_act), call
        assert torch.equal(pm.u_prev, ref_u_prev), call
        assert int(pm.naninf_chunks.item()) == ref_naninf
        assert pm.predictions.shape == (B, T, 14)
        u_prev = ref_u_prev


def test_actor_gradient_reaches_the_policy_output():
    B = 12
    rng = np.random.default_rng(5)
    inp = wl.make_inputs(B, T, seed=7)
    states = torch.from_numpy(inp["x0"]).to(DEV)
    sc = torch.from_numpy((1 / (1 + np.exp(-rng.normal(0, 1.5, (B, 28 * T))))).astype(np.float32)).to(DEV)
    sc.requires_grad_(True)
    pm = policy_mpc.PolicyMPC(T, DT, lqr_iter=2, eps=0.1, device=DEV)
    act = pm.actor(sc, states)
    act.sum().backward()
    assert sc.grad is not None and torch.isfinite(sc.grad).all() and sc.grad.abs().sum() > 0
    pm_stop = policy_mpc.PolicyMPC(T, DT, lqr_iter=2, eps=0.1, grad_mode="stop", device=DEV)
    act2 = pm_stop.actor(sc, states)
    assert not act2.requires_grad


def test_actor_fastmpc_numerics_matches_chunked_loop():
    """PolicyMPC(numerics="fastmpc"): with fewer than four iterations the batch
    stop is never read early, so the elements are independent and the one-call
    actor equals the chunked loop on the FastMPC numerics."""
    B = 21
    rng = np.random.default_rng(9)
    inp = wl.make_inputs(B, T, seed=10)
    states = torch.from_numpy(inp["x0"]).to(DEV)
    pm = policy_mpc.PolicyMPC(T, DT, lqr_iter=3, eps=0.1, chunk=8, device=DEV, numerics="fastmpc")
    assert pm.solver.numerics == "fastmpc"
    sc = torch.from_numpy((1 / (1 + np.exp(-rng.normal(0, 1.5, (B, 28 * T))))).astype(np.float32)).to(DEV)
    u_prev = torch.zeros(B, 4, device=DEV)
    u_prev[:, 0] = MASS * 9.8066
    with torch.no_grad():
        act = pm.actor(sc, states)
    ref_act, ref_u_prev, _ = _reference_loop(sc, states, u_prev, 8, 3, 0.1, numerics="fastmpc")
    assert torch.equal(act, ref_act)
    assert torch.equal(pm.u_prev, ref_u_prev)

