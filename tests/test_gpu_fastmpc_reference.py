"""The FastMPC numerics mode against the reference's own CUDA kernels.

oracle/fastmpc_ref_cuda.py re-executes the reference FastMPC extension's CUDA build
on the GPU: its kernels, compiled from the reference sources with its own
flags (--use_fast_math) into oracle/_ref/, driven by a torch restatement of
its host loop. The B200 solve records its line-search decisions and batch
stop; the re-executed reference replays them, and X, U must agree to 1e-4
(relative to the element's largest magnitude), the tight masks on 99 % of
entries, and the gradients of x0, C, c to 1e-3. The cases use the FastMPC
operator's zero terminal cost and references, as the operator does.
"""

import numpy as np
import pytest
import torch

from oracle import fastmpc_ref_cuda as ref
import ilqr_native as nat
import ilqr_workload as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref.available(),
                                 reason="oracle/_ref/libfastmpc_ref.so not built (needs the reference sources)")]
DEV = "cuda"
LO = np.array([0.0, -10.0, -10.0, -4.0], np.float32)
HI = np.array([34.0, 10.0, 10.0, 4.0], np.float32)


def _t(a):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, torch.float32)


def _rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    ax = tuple(range(1, a.ndim))
    scale = np.maximum(np.abs(b).max(axis=ax, keepdims=True), 1.0)
    return (np.abs(a - b) / scale).max(axis=ax)


def _case(name):
    if name == "cfg1_b16_t5":
        return wl.make_inputs(16, 5, seed=0), True, 10
    if name == "cfg2_b64_t10":
        return wl.make_inputs(64, 10, seed=1), True, 10
    if name == "cfg3_b48_t20":
        return wl.make_inputs(48, 20, seed=2), True, 5
    if name == "dense_b8_t6":
        d = wl.make_inputs(8, 6, seed=3)
        extra = wl.make_dense_costs(8, 6, seed=4)
        return dict(d, C=extra["C"], c=extra["c"]), True, 6
    if name == "nobox_b8_t5":
        return wl.make_inputs(8, 5, seed=5), False, 5
    if name == "ragged_b13_t7":
        return wl.make_inputs(13, 7, seed=6, r=15.0), True, 9
    if name == "cfg5_b8_t50":
        return wl.make_inputs(8, 50, seed=7, r=15.0), True, 8
    raise KeyError(name)


# cfg5_b8_t50 (long horizon) is checked against the problem's conditioning instead
CASES = ["cfg1_b16_t5", "cfg2_b64_t10", "cfg3_b48_t20", "dense_b8_t6", "nobox_b8_t5", "ragged_b13_t7"]


@pytest.mark.parametrize("name", CASES)
def test_fastmpc_matches_reference_kernels(name):
    d, boxed, iters = _case(name)
    lo, hi = (_t(LO), _t(HI)) if boxed else (None, None)
    ours = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=lo, u_max=hi, dt=0.05,
                             max_iter=iters, want_trace=True)
    run = int(ours["batch_info"][1])
    r = ref.solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), lo, hi, dt=0.05, max_iter=iters,
                  forced=ours["trace"].long(), forced_stop=run)
    assert r["iters"] == run
    for k in ("X", "U"):
        err = _rel(ours[k], r[k])
        assert err.max() <= 1e-4, (k, float(err.max()), int(err.argmax()))
    agree = (ours["tight"].bool() == r["tight"]).float().mean().item()
    assert agree >= 0.99, agree
    # the backward at each side's own solution
    B, T = d["U_init"].shape[:2]
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    g = nat.fastmpc_backward(ours["X"], ours["U"], ours["X_lin"], ours["U_lin"], _t(d["C"]), gX, gU,
                             tight=ours["tight"] if boxed else None, dt=0.05)
    rg = ref.backward(r, gX, gU)
    for k in ("x0", "C", "c"):
        err = _rel(g[k], rg[k])
        assert err.max() <= 1e-3, (k, float(err.max()), int(err.argmax()))


def test_long_horizon_within_conditioning():
    """T = 50, targets at 15 m, 8 iterations, against the reference kernels
    replaying the B200 solve's decisions. Per element, X, U and the gradients
    agree to the plain bars or to CONDITION_FACTOR times the oracle's own
    response to 1e-7 noise in C, whichever is larger."""
    from parity import CONDITION_FACTOR, fm_condition_spread
    d, boxed, iters = _case("cfg5_b8_t50")
    ours = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                             dt=0.05, max_iter=iters, want_trace=True)
    run = int(ours["batch_info"][1])
    r = ref.solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), _t(LO), _t(HI), dt=0.05, max_iter=iters,
                  forced=ours["trace"].long(), forced_stop=run)
    assert r["iters"] == run
    B, T = d["U_init"].shape[:2]
    gXn, gUn = wl.make_backward_seeds(B, T)
    sp = fm_condition_spread(d, ours["trace"].long().cpu().numpy(), run, LO, HI, 0.05, iters, grad_seeds=(gXn, gUn))
    g = nat.fastmpc_backward(ours["X"], ours["U"], ours["X_lin"], ours["U_lin"], _t(d["C"]), _t(gXn), _t(gUn),
                             tight=ours["tight"], dt=0.05)
    rg = ref.backward(r, _t(gXn), _t(gUn))
    pairs = [("X", ours["X"], r["X"], 1e-4), ("U", ours["U"], r["U"], 1e-4)]
    pairs += [(k, g[k], rg[k], 1e-3) for k in ("x0", "C", "c")]
    for k, a, b_, tol in pairs:
        err = _rel(a, b_)
        bad = np.nonzero(err > np.maximum(tol, CONDITION_FACTOR * sp[k]))[0]
        assert bad.size == 0, (k, [(int(i), float(err[i]), float(sp[k][i])) for i in bad])


@pytest.mark.parametrize("name", ["cfg1_b16_t5", "cfg2_b64_t10", "cfg3_b48_t20"])
def test_free_run_parts_from_reference_only_at_ties(name):
    """Without replay each side decides for itself. An element whose decisions
    match the reference's ends within 1e-4 of it; where they part, the first
    differing decision is a near-tie in the reference's own costs: two step
    sizes within 1e-5 of each other (relative), or an accept/reject call on an
    improvement below 1e-5 of the cost."""
    d, boxed, iters = _case(name)
    ours = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                             dt=0.05, max_iter=iters, want_trace=True)
    r = ref.solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), _t(LO), _t(HI), dt=0.05, max_iter=iters)
    n = min(int(ours["batch_info"][1]), r["iters"])
    to = ours["trace"][:, :n].long().cpu().numpy()
    tr = r["trace"][:, :n].cpu().numpy()
    costs = r["costs"][:, :n].double().cpu().numpy()
    best = r["best_before"][:, :n].double().cpu().numpy()
    err = _rel(ours["U"], r["U"])
    parted = 0
    for b in range(to.shape[0]):
        diff = np.nonzero(to[b] != tr[b])[0]
        if diff.size == 0:
            if int(ours["batch_info"][1]) == r["iters"]:
                assert err[b] <= 1e-4, (b, err[b])
            continue
        parted += 1
        i = diff[0]
        c = costs[b, i]
        scale = max(np.abs(c).max(), abs(best[b, i]), 1e-30)
        jo, jr = to[b, i], tr[b, i]
        if jo >= 0 and jr >= 0:
            gap = abs(c[jo] - c[jr])
        else:
            j = jo if jo >= 0 else jr
            gap = abs(c[j] - best[b, i]) if j >= 0 else abs(c[-jo - 1] - c[-jr - 1])
        assert gap <= 1e-5 * scale, (b, i, jo, jr, gap / scale)
    assert parted < to.shape[0]


def test_pnqp4_batch_matches_reference_kernel():
    """drone_pnqp4_batch against the reference's own PNQP-4 kernel on the
    golden problems (mpc.pytorch pnqp's set) and on the box QPs of a solve:
    the same optimum to 1e-4 and the same free mask, cold and warm started."""
    import os
    from parity import GOLDEN_DIR
    d = np.load(os.path.join(GOLDEN_DIR, "pnqp4_n256.npz"))
    H, q, lo, hi = (_t(d[k]) for k in ("H", "q", "lower", "upper"))
    for x_init in (None, _t(d["opt_x"].astype(np.float32))):
        x, fm = nat.pnqp4_batch(H, q, lo, hi, x_init)
        rx, rfm = ref.pnqp4_batch(H, q, lo, hi, x_init)
        scale = torch.clamp(rx.abs().amax(1, keepdim=True), min=1.0)
        close = ((x - rx).abs() / scale).amax(1) <= 1e-4
        assert close.float().mean().item() >= 0.98, close.float().mean().item()
        assert torch.equal(fm[close], rfm[close])



def _rand_lqr(B, T, seed):
    rng = np.random.default_rng(seed)
    A = np.eye(10) + 0.05 * rng.normal(size=(B, T, 10, 10))
    Bm = 0.1 * rng.normal(size=(B, T, 10, 4))
    G = rng.normal(size=(B, T, 14, 14)) * 0.3
    C = G @ np.swapaxes(G, -1, -2) / 14 + np.eye(14) * rng.uniform(0.5, 2.0, (B, T, 14))[..., None]
    GN = rng.normal(size=(B, 10, 10)) * 0.3
    f = lambda a: _t(np.asarray(a, np.float32))
    return dict(A=f(A), B=f(Bm), l_xx=f(C[..., :10, :10]), l_uu=f(C[..., 10:, 10:]), l_xu=f(C[..., :10, 10:]),
                l_x=f(rng.normal(size=(B, T, 10))), l_u=f(rng.normal(size=(B, T, 4))),
                l_xxN=f(GN @ np.swapaxes(GN, -1, -2) / 10), l_xN=f(rng.normal(size=(B, 10))),
                tight=torch.as_tensor(rng.uniform(size=(B, T, 4)) < 0.3, device=DEV))


def test_extension_entry_points_match_reference_kernels():
    """The FastMPC extension surface's separate entry points (Jacobian, masked
    adjoint Riccati, assembly) against the reference kernels they replace."""
    from oracle import fastmpc_ref_cuda as fastmpc_ref
    B, T = 24, 7
    rng = np.random.default_rng(3)
    X = np.zeros((B, T + 1, 10), np.float32)
    X[..., :3] = rng.normal(size=(B, T + 1, 3))
    q = rng.normal(size=(B, T + 1, 4))
    X[..., 3:7] = q / np.linalg.norm(q, axis=-1, keepdims=True)
    X[..., 7:] = rng.normal(size=(B, T + 1, 3))
    U = np.concatenate([rng.uniform(0, 30, (B, T, 1)), rng.normal(size=(B, T, 3))], -1).astype(np.float32)
    Xt, Ut = _t(X), _t(U)
    A, Bm = nat.fastmpc_linearize(Xt, Ut, 0.05)
    rA = torch.empty(B * T, 10, 10, device=DEV)
    rB = torch.empty(B * T, 10, 4, device=DEV)
    xn = torch.empty(B * T, 10, device=DEV)
    L = fastmpc_ref.lib()
    p = fastmpc_ref._p
    assert L.fmref_step_jacobian(p(Xt[:, :T].reshape(-1, 10).contiguous()), p(Ut.reshape(-1, 4).contiguous()), p(xn),
                                 p(rA), p(rB), 0.05, B * T, fastmpc_ref._s()) == 0
    assert torch.allclose(A, rA.view(B, T, 10, 10), rtol=1e-5, atol=1e-6)
    assert torch.allclose(Bm, rB.view(B, T, 10, 4), rtol=1e-5, atol=1e-6)
    d = _rand_lqr(B, T, 4)
    for tight in (None, d["tight"]):
        K, k, v0 = nat.fastmpc_adjoint_lqr(d["A"], d["B"], d["l_xx"], d["l_uu"], d["l_xu"], d["l_x"], d["l_u"],
                                           d["l_xxN"], d["l_xN"], None if tight is None else tight.to(torch.uint8))
        rK, rk, rv = (torch.zeros(B, T, 4, 10, device=DEV), torch.zeros(B, T, 4, device=DEV),
                      torch.zeros(B, 10, device=DEV))
        tm = None if tight is None else tight.to(torch.uint8).contiguous()
        assert L.fmref_riccati(p(d["A"]), p(d["B"]), p(d["l_xx"]), p(d["l_uu"]), p(d["l_xu"]), p(d["l_x"]),
                               p(d["l_u"]), p(d["l_xxN"]), p(d["l_xN"]), p(tm), 1e-6, B, T, p(rK), p(rk), p(rv),
                               fastmpc_ref._s()) == 0
        for a, b_ in ((K, rK), (k, rk), (v0, rv)):
            assert _rel(a, b_).max() <= 1e-4
        g = nat.fastmpc_assembly(K, k, v0, d["A"], d["B"], Xt, Ut, None, None, True, True, True, True)
        z = lambda *s: torch.zeros(*s, device=DEV)
        rg = [z(B, T, 14, 14), z(B, T, 14), z(B, 10), z(B, T + 1, 10), z(B, T, 4), z(B, 14, 14), z(B, 14)]
        assert L.fmref_assembly(p(K), p(k), p(v0), p(d["A"]), p(d["B"]), p(Xt), p(Ut), p(z(B, T + 1, 10)),
                                p(z(B, T, 4)), *[p(r_) for r_ in rg], B, T, fastmpc_ref._s()) == 0
        for a, b_ in zip(g, rg):
            assert _rel(a, b_).max() <= 1e-5


def test_extension_object_fastmpc_numerics():
    """load_drone_ilqr_ext(numerics="fastmpc"): drone_ilqr_solve returns the
    fused solve's X, U, tight mask and the Jacobian at its last linearisation
    point; the operator-style backward through its separate entry points
    agrees with the fused backward."""
    import drone_ilqr
    d, _, iters = _case("cfg1_b16_t5")
    B, T = d["U_init"].shape[:2]
    ext = drone_ilqr.load_drone_ilqr_ext(numerics="fastmpc")
    assert ext.numerics == "fastmpc" and drone_ilqr.load_drone_ilqr_ext().numerics == "diffmpc"
    z = lambda *s: torch.zeros(*s, device=DEV)
    res = ext.drone_ilqr_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), z(B, 14, 14), z(B, 14),
                               z(B, T + 1, 10), z(B, T, 4), _t(LO), _t(HI), 0.05, iters, 1e-6, 1e-6)
    X, U, l_xx, l_uu, l_xu, l_xxN, A_lin, B_lin, tight, converged = res
    o = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                          dt=0.05, max_iter=iters)
    assert torch.equal(X, o["X"]) and torch.equal(U, o["U"]) and torch.equal(tight, o["tight"].bool())
    A2, B2 = nat.fastmpc_linearize(o["X_lin"], o["U_lin"], 0.05)
    assert torch.equal(A_lin, A2) and torch.equal(B_lin, B2)
    assert converged == bool(int(o["batch_info"][0]))
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    K, k, v0 = ext.drone_backward_pass_batched(A_lin, B_lin, l_xx, l_uu, l_xu, -gX[:, :T], -gU, l_xxN, -gX[:, -1],
                                               tight, 1e-6)
    gC, gc, gx0, *_ = ext.drone_implicit_diff_assembly(K, k, v0, A_lin, B_lin, X, U, z(B, T + 1, 10), z(B, T, 4))
    g = nat.fastmpc_backward(o["X"], o["U"], o["X_lin"], o["U_lin"], _t(d["C"]), gX, gU, tight=o["tight"], dt=0.05)
    for a, b_ in ((gx0, g["x0"]), (gC, g["C"]), (gc, g["c"])):
        assert _rel(a, b_).max() <= 1e-5
