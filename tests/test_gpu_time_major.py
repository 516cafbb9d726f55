"""The time-major cost layout ([T,B,...], the layout QuadCost carries in
mpc.pytorch and the reference's operators) against the batch-major one: the
kernels read C, c and write grad_C, grad_c through per-element and per-step
strides, so the two entry points must agree bit for bit on every output, for
both models, dense costs with every optional input, and ragged batches."""

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl
import mpc_compat

pytestmark = pytest.mark.gpu
DEV = "cuda"
ALL_GRADS = ("x0", "C", "c", "C_final", "c_final", "x_ref", "u_ref")


def _t(a):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, torch.float32)


def _tm(a):
    return a.transpose(0, 1).contiguous()


def _inputs(model, B, T, dense):
    if model == 13:
        d = wl.make_rotor13_inputs(B, T, seed=3)
        nx, n, lo, hi = wl.NX13, wl.N13, wl.U_MIN13, wl.U_MAX13
    else:
        d = wl.make_inputs(B, T, seed=3)
        nx, n, lo, hi = wl.NX, wl.N, None, None
    inp = dict(x0=_t(d["x0"]), U_init=_t(d["U_init"]), C=_t(d["C"]), c=_t(d["c"]))
    opt = dict(C_final=None, c_final=None, x_ref=None, u_ref=None)
    if dense:
        rng = np.random.default_rng(11)
        G = rng.normal(size=(B, T, n, n)).astype(np.float32) * 0.2
        inp["C"] = inp["C"] + _t(G @ np.swapaxes(G, -1, -2) / n)
        inp["c"] = inp["c"] + _t(rng.normal(0.0, 1.0, (B, T, n)))
        Gf = rng.normal(size=(B, n, n)).astype(np.float32) * 0.3
        opt = dict(C_final=_t(Gf @ np.swapaxes(Gf, -1, -2) / n), c_final=_t(rng.normal(0.0, 1.0, (B, n))),
                   x_ref=_t(rng.normal(0.0, 0.05, (B, T + 1, nx))), u_ref=_t(rng.normal(0.0, 0.05, (B, T, 4))))
    box = dict(u_min=_t(lo), u_max=_t(hi)) if model == 13 else dict(
        u_min=_t(np.array([0.0, -3.0, -3.0, -3.0])), u_max=_t(np.array([20.0, 3.0, 3.0, 3.0])))
    gX, gU = wl.make_backward_seeds(B, T, nx=nx)
    return inp, opt, box, _t(gX), _t(gU)


@pytest.mark.parametrize("model,B,T,dense", [(10, 37, 7, True), (10, 3000, 20, False), (13, 37, 7, True),
                                             (13, 700, 20, False)])
def test_time_major_entry_points_equal_batch_major(model, B, T, dense):
    inp, opt, box, gX, gU = _inputs(model, B, T, dense)
    solve = nat.rotor13_solve if model == 13 else nat.solve
    backward = nat.rotor13_backward if model == 13 else nat.backward
    kw = dict(dt=0.05, max_iter=5, reg_eps=1e-6, want_trace=True, want_stats=True, **box)
    ref = solve(inp["x0"], inp["U_init"], inp["C"], inp["c"], **opt, **kw)
    got = solve(inp["x0"], inp["U_init"], _tm(inp["C"]), _tm(inp["c"]), **opt, time_major=True, **kw)
    for k in ref:
        assert torch.equal(torch.nan_to_num(got[k]), torch.nan_to_num(ref[k])), k
    bkw = dict(C_final=opt["C_final"], x_ref=opt["x_ref"], u_ref=opt["u_ref"], tight=ref["tight"], dt=0.05,
               reg_eps=1e-6, need=ALL_GRADS)
    rg = backward(ref["X"], ref["U"], inp["C"], gX, gU, **bkw)
    gg = backward(ref["X"], ref["U"], _tm(inp["C"]), gX, gU, time_major=True, **bkw)
    for k in ALL_GRADS:
        want = _tm(rg[k]) if k in ("C", "c") else rg[k]
        assert torch.equal(gg[k], want), k


@pytest.mark.parametrize("n_state", [10, 13])
def test_operator_broadcast_costs_equal_full_costs(n_state):
    """FastMPC passes QuadCost's [T,B,...] tensors to the kernels as they are;
    a shared C [n,n], c [n] gives the solution and, summed over steps and
    elements, the gradients of the same costs given in full."""
    B, T = 24, 6
    n = n_state + 4
    rng = np.random.default_rng(5)
    G = rng.normal(size=(n, n)).astype(np.float32) * 0.3
    C2 = _t(G @ G.T / n + np.eye(n, dtype=np.float32))
    c1 = _t(rng.normal(0.0, 1.0, n))
    inp, _, box, gX, gU = _inputs(n_state, B, T, dense=False)
    lo = box["u_min"].expand(T, B, 4)
    hi = box["u_max"].expand(T, B, 4)
    dx = type("Dx", (), {"dt": 0.05})()
    outs = []
    for full in (False, True):
        C = (C2.expand(T, B, n, n).contiguous() if full else C2.clone()).requires_grad_(True)
        c = (c1.expand(T, B, n).contiguous() if full else c1.clone()).requires_grad_(True)
        x0 = inp["x0"].clone().requires_grad_(True)
        m = mpc_compat.FastMPC(n_state, 4, T, u_lower=lo, u_upper=hi, lqr_iter=5, eps=1e-6)
        X, U, _ = m(x0, mpc_compat.QuadCost(C, c), dx)
        ((X * _tm(gX)).sum() + (U * _tm(gU)).sum()).backward()
        outs.append((X.detach(), U.detach(), x0.grad, C.grad, c.grad))
    (Xb, Ub, gxb, gCb, gcb), (Xf, Uf, gxf, gCf, gcf) = outs
    assert torch.equal(Xb, Xf) and torch.equal(Ub, Uf)
    assert torch.equal(gxb, gxf)
    assert torch.allclose(gCb, gCf.sum((0, 1)), rtol=1e-5, atol=1e-5 * float(gCf.abs().sum((0, 1)).max()))
    assert torch.allclose(gcb, gcf.sum((0, 1)), rtol=1e-5, atol=1e-5 * float(gcf.abs().sum((0, 1)).max()))
