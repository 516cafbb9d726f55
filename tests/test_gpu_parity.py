"""GPU parity of the CUDA solver (through the C ABI) against the reference's
golden vectors and the CPU oracle. Bars: 1e-4 on X, U and 1e-3 on gradients
(per-element norm-wise relative error, tests/parity.py)."""

import os

import numpy as np
import pytest
import torch

import drone_ilqr
import ilqr_native as nat
import ilqr_workload as wl
import mpc_compat
import oracle as O
from parity import (GOLDEN_DIR, GRAD_KEYS, STRICT_CASES, TOL_GRAD, TOL_XU, case_kwargs, certify_ties, load,
                    max_rel, same_decisions)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
KEYMAP = {"grad_x0": "x0", "grad_C": "C", "grad_c": "c", "grad_C_final": "C_final",
          "grad_c_final": "c_final", "grad_xref": "x_ref", "grad_uref": "u_ref"}


def g(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, dtype)


def gpu_solve(d, forced=None, **over):
    kw = case_kwargs(d)
    kw.update(over)
    out = nat.solve(g(d["x0"]), g(d["U_init"]), g(d["C"]), g(d["c"]), g(kw["C_f"]), g(kw["c_f"]),
                    g(kw["x_ref"]), g(kw["u_ref"]), g(kw["u_min"]), g(kw["u_max"]), dt=kw["dt"],
                    max_iter=kw["max_iter"], reg_eps=kw["reg"], alphas=kw["alphas"],
                    forced_trace=g(forced, torch.int8), want_trace=True, want_stats=True)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}, kw


def gpu_backward(d, X, U, tight, kw, gX=None, gU=None):
    need = tuple(KEYMAP.values())
    out = nat.backward(g(X), g(U), g(d["C"]), g(d["gX"] if gX is None else gX),
                       g(d["gU"] if gU is None else gU), C_final=g(kw["C_f"]), x_ref=g(kw["x_ref"]),
                       u_ref=g(kw["u_ref"]), tight=g(tight, torch.uint8), dt=kw["dt"],
                       reg_eps=kw["reg"], need=need)
    torch.cuda.synchronize()
    return {gk: out[nk].cpu().numpy() for gk, nk in KEYMAP.items()}


def test_dynamics_and_linearize_match_reference():
    d = load("dynamics_n64")
    xn = nat.dynamics(g(d["x"]), g(d["u"]), float(d["dt"])).cpu().numpy()
    assert max_rel(xn, d["x_next"]) <= 4e-7
    X = np.concatenate([d["x"][:, None], np.zeros_like(d["x"])[:, None]], 1)
    A, Bm = nat.linearize(g(X), g(d["u"][:, None]), float(d["dt"]))
    assert max_rel(A.cpu().numpy()[:, 0], d["A"]) <= 1e-6
    assert max_rel(Bm.cpu().numpy()[:, 0], d["B"]) <= 1e-6


@pytest.mark.parametrize("name", STRICT_CASES)
def test_replay_matches_reference(name):
    """Replaying the reference's decisions: X, U within 1e-4, tight mask
    identical, gradients at the solution within 1e-3."""
    d = load(name)
    r, kw = gpu_solve(d, forced=d["ref_trace"])
    assert max_rel(r["X"], d["ref_X"]) <= TOL_XU
    assert max_rel(r["U"], d["ref_U"]) <= TOL_XU
    assert np.array_equal(r["tight"].astype(bool), d["ref_tight"])
    gr = gpu_backward(d, r["X"], r["U"], r["tight"], kw)
    for k in GRAD_KEYS:
        assert max_rel(gr[k], d["ref_" + k]) <= TOL_GRAD, k


@pytest.mark.parametrize("name", STRICT_CASES)
def test_backward_at_reference_solution(name):
    d = load(name)
    kw = case_kwargs(d)
    gr = gpu_backward(d, d["ref_X"], d["ref_U"], d["ref_tight"].astype(np.uint8), kw)
    for k in GRAD_KEYS:
        assert max_rel(gr[k], d["ref_" + k]) <= TOL_GRAD, k


@pytest.mark.parametrize("name", STRICT_CASES)
def test_free_run(name):
    """Free-running GPU solve: (a) the oracle replaying the GPU's own decisions
    reproduces its X, U within 1e-4; (b) every decision where the GPU parts
    from the reference is an fp32 tie in the reference's candidate costs;
    (c) elements that never part match the reference within 1e-4."""
    d = load(name)
    r, kw = gpu_solve(d)
    o = O.solve(d["x0"], d["U_init"], d["C"], d["c"], forced=r["trace"], **kw)
    assert max_rel(r["X"], o["X"]) <= TOL_XU
    assert max_rel(r["U"], o["U"]) <= TOL_XU
    n_div, fails = certify_ties(r["trace"], d)
    assert not fails, fails
    same = same_decisions(r["trace"], d["ref_trace"])
    assert max_rel(r["X"][same], d["ref_X"][same]) <= TOL_XU
    assert max_rel(r["U"][same], d["ref_U"][same]) <= TOL_XU
    conv = nat.converged_flag(torch.tensor(r["stall_iter"]), torch.tensor(r["stall_gap"]),
                              torch.tensor(r["status"]), kw["max_iter"], 1e-6)
    ref_conv = O.global_converged_flag(o["stall_iter"], o["stall_gap"], kw["max_iter"], 1e-6, True)
    assert conv == ref_conv


def test_chol_fallback_path():
    d = load("indef_b8_t4")
    r, _ = gpu_solve(d, forced=d["ref_trace"])
    assert (r["status"][::2] & 1).all() and not (r["status"][1::2] & 1).any()


def test_long_horizon_never_improving_elements_exact():
    d = load("cfg5_b64_t50")
    r, _ = gpu_solve(d, forced=d["ref_trace"])
    never = d["ref_trace"].max(axis=1) < 0
    assert max_rel(r["X"][never], d["ref_X"][never]) <= 1e-6
    assert np.array_equal(r["U"][never], d["ref_U"][never])


def test_long_horizon_within_conditioning():
    """T=50, 15 m targets, every element, replaying the reference's decisions.
    Where the problem is well conditioned (CONDITION_FACTOR times the oracle's
    own response to 1e-7 noise in C stays below COND_CAP), X, U and the
    gradients at the GPU's solution agree with the reference to the plain bars
    or to that multiple of the response, per element. Where it does not, one
    ulp of noise moves the answer by more than COND_CAP, so no fp32 run pins
    another: those elements are not compared with the reference's fp32 run but
    with the oracle's fp64 replay of the same decisions, and the GPU's error
    there must stay within ROUNDING_FACTOR times the larger fp32 error of the
    two other realisations of the same arithmetic (the reference's fp32 run
    and the oracle's)."""
    from parity import CONDITION_FACTOR, diffmpc_condition_spread, rel_per_elem
    COND_CAP, ROUNDING_FACTOR = 0.05, 30.0
    d = load("cfg5_b64_t50")
    r, kw = gpu_solve(d, forced=d["ref_trace"])
    gg = gpu_backward(d, r["X"], r["U"], r["tight"], kw)
    sp = diffmpc_condition_spread(d, d["ref_trace"])
    o32 = O.solve(d["x0"], d["U_init"], d["C"], d["c"], forced=d["ref_trace"], **kw)
    o64 = O.solve(d["x0"], d["U_init"], d["C"], d["c"], forced=d["ref_trace"], dtype=np.float64, **kw)
    pairs = [("X", r["X"], TOL_XU), ("U", r["U"], TOL_XU)] + [(k, gg[k], TOL_GRAD) for k in GRAD_KEYS]
    ill = np.zeros(len(d["x0"]), bool)
    for k, a, tol in pairs:
        ill |= CONDITION_FACTOR * sp[k] > COND_CAP
    for k, a, tol in pairs:
        err = rel_per_elem(a, d["ref_" + k])
        bad = np.nonzero(~ill & (err > np.maximum(tol, CONDITION_FACTOR * sp[k])))[0]
        assert bad.size == 0, (k, [(int(b), float(err[b]), float(sp[k][b])) for b in bad])
    for k in ("X", "U"):
        e_gpu = rel_per_elem(r[k], o64[k])
        e_o32 = np.maximum(rel_per_elem(o32[k], o64[k]), rel_per_elem(d["ref_" + k], o64[k]))
        bad = np.nonzero(ill & (e_gpu > np.maximum(TOL_XU, ROUNDING_FACTOR * e_o32)))[0]
        assert bad.size == 0, (k, [(int(b), float(e_gpu[b]), float(e_o32[b])) for b in bad])


def _dx():
    return type("Dx", (), {"dt": wl.DT})()


def test_fastmpc_autograd_end_to_end():
    """FastMPC(...)(x_init, QuadCost(C, c), dx) with autograd: outputs equal
    the direct solve, gradients match the oracle backward at the GPU's
    solution, and the layouts are mpc.pytorch's [T, B, ...]."""
    d = load("cfg1_b16_t5")
    B, T = d["x0"].shape[0], d["U_init"].shape[1]
    x0 = g(d["x0"]).requires_grad_(True)
    C = g(d["C"]).permute(1, 0, 2, 3).contiguous().requires_grad_(True)
    c = g(d["c"]).permute(1, 0, 2).contiguous().requires_grad_(True)
    lo = g(np.broadcast_to(wl.U_MIN, (T, 1, 4)).copy())
    hi = g(np.broadcast_to(wl.U_MAX, (T, 1, 4)).copy())
    m = mpc_compat.MPC(10, 4, T, u_lower=lo, u_upper=hi, lqr_iter=int(d["max_iter"]), eps=1e-6)
    x, u, objs = m(x0, mpc_compat.QuadCost(C, c), _dx())
    assert x.shape == (T + 1, B, 10) and u.shape == (T, B, 4) and objs.shape == (T, B)
    gX = g(d["gX"]).permute(1, 0, 2)
    gU = g(d["gU"]).permute(1, 0, 2)
    ((x * gX).sum() + (u * gU).sum()).backward()
    r, kw = gpu_solve(d)
    assert np.array_equal(x.detach().permute(1, 0, 2).cpu().numpy(), r["X"])
    assert np.array_equal(u.detach().permute(1, 0, 2).cpu().numpy(), r["U"])
    o = O.backward(r["X"], r["U"], d["C"], None, None, None, r["tight"], d["gX"], d["gU"],
                   kw["dt"], kw["reg"])
    assert max_rel(x0.grad.cpu().numpy(), o["grad_x0"]) <= TOL_GRAD
    assert max_rel(C.grad.permute(1, 0, 2, 3).cpu().numpy(), o["grad_C"]) <= TOL_GRAD
    assert max_rel(c.grad.permute(1, 0, 2).cpu().numpy(), o["grad_c"]) <= TOL_GRAD
    with torch.no_grad():
        x2, u2, _ = m(x0, mpc_compat.QuadCost(C, c), _dx())
    assert torch.equal(x2, x.detach()) and torch.equal(u2, u.detach())


def test_extension_surface():
    """load_drone_ilqr_ext(): drone_ilqr_solve's 10-tuple, and the explicit-A/B
    backward pair agreeing with the fused backward."""
    d = load("cfg2_b32_t10")
    B, T = d["x0"].shape[0], d["U_init"].shape[1]
    ext = drone_ilqr.load_drone_ilqr_ext()
    z = lambda *s: torch.zeros(*s, device=DEV)
    res = ext.drone_ilqr_solve(g(d["x0"]), g(d["U_init"]), g(d["C"]), g(d["c"]), z(B, 14, 14),
                               z(B, 14), z(B, T + 1, 10), z(B, T, 4), g(wl.U_MIN), g(wl.U_MAX),
                               wl.DT, int(d["max_iter"]), 1e-6, 1e-6)
    X, U, l_xx, l_uu, l_xu, l_xxN, A, Bm, tight, conv = res
    assert X.shape == (B, T + 1, 10) and U.shape == (B, T, 4)
    assert l_xx.shape == (B, T, 10, 10) and l_uu.shape == (B, T, 4, 4) and l_xu.shape == (B, T, 10, 4)
    assert l_xxN.shape == (B, 10, 10) and A.shape == (B, T, 10, 10) and Bm.shape == (B, T, 10, 4)
    assert tight.dtype == torch.bool and isinstance(conv, bool)
    r, kw = gpu_solve(d)
    assert np.array_equal(X.cpu().numpy(), r["X"])
    gX, gU = g(d["gX"]), g(d["gU"])
    K, k, v0 = ext.drone_backward_pass_batched(A, Bm, l_xx, l_uu, l_xu, -gX[:, :T], -gU, l_xxN,
                                               -gX[:, -1], tight, 1e-6)
    gC, gc, gx0, gxr, gur, gCf, gcf = ext.drone_implicit_diff_assembly(
        K, k, v0, A, Bm, X, U, z(B, T + 1, 10), z(B, T, 4), True, True, True, True)
    fused = gpu_backward(d, r["X"], r["U"], r["tight"], kw)
    assert max_rel(gC.cpu().numpy(), fused["grad_C"]) <= TOL_GRAD
    assert max_rel(gc.cpu().numpy(), fused["grad_c"]) <= TOL_GRAD
    assert max_rel((-v0).cpu().numpy(), fused["grad_x0"]) <= TOL_GRAD
    assert max_rel(gxr.cpu().numpy(), fused["grad_xref"]) <= TOL_GRAD
    assert max_rel(gCf.cpu().numpy(), fused["grad_C_final"]) <= TOL_GRAD


def test_batch_not_multiple_of_warp_and_prefix_independence():
    """Elements are independent: the first 16 elements of a B=45 solve are
    bit-identical to a B=16 solve; padding lanes never write."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=45)
    d45 = dict(inp, bounds=np.array(True), dt=np.array(wl.DT), max_iter=np.array(5),
               reg=np.array(1e-6), alphas=np.array(cfg["alphas"], np.float32))
    d16 = {k: (v[:16] if isinstance(v, np.ndarray) and v.ndim > 1 else v) for k, v in d45.items()}
    r45, _ = gpu_solve(d45)
    r16, _ = gpu_solve(d16)
    for k in ("X", "U", "tight", "trace"):
        assert np.array_equal(r45[k][:16], r16[k]), k


def test_invalid_inputs_raise():
    d = load("b1_t1")
    with pytest.raises(RuntimeError, match="shape"):
        nat.solve(g(d["x0"]), g(d["U_init"]), g(d["C"])[:, :, :13], g(d["c"]))
    with pytest.raises(RuntimeError, match="float32"):
        nat.solve(g(d["x0"]).double(), g(d["U_init"]), g(d["C"]), g(d["c"]))
    C = torch.empty(1 * 1 * 14 * 14 + 1, device=DEV)[1:].view(1, 1, 14, 14)
    C.copy_(g(d["C"]))
    with pytest.raises(RuntimeError, match="aligned"):
        nat.solve(g(d["x0"]), g(d["U_init"]), C, g(d["c"]))
    with pytest.raises(RuntimeError, match="step sizes"):
        nat.solve(g(d["x0"]), g(d["U_init"]), g(d["C"]), g(d["c"]), alphas=())


def test_nonfinite_elements_are_isolated():
    """A NaN in one element's x0 and an infinite cost weight in another's C:
    both reject their first step as the reference does (objective NaN / inf,
    never improved), keep U_init and their initial rollout, and are flagged
    non-finite where X is; every other element of the batch (warp-mates
    included) is bit-identical to the run without them."""
    d = load("cfg1_b16_t5")
    bad = dict(d)
    bad["x0"] = d["x0"].copy()
    bad["x0"][3, 0] = np.nan
    bad["C"] = d["C"].copy()
    bad["C"][7, 2, 1, 1] = np.inf
    r, kw = gpu_solve(bad)
    r0, _ = gpu_solve(d)
    with np.errstate(invalid="ignore", over="ignore"):
        o = O.solve(bad["x0"], d["U_init"], bad["C"], d["c"], **kw)
    others = [b for b in range(16) if b not in (3, 7)]
    for k in ("X", "U", "tight", "trace"):
        assert np.array_equal(r[k][others], r0[k][others]), k
    for b in (3, 7):
        assert r["trace"][b, 0] < 0 and (r["trace"][b, 1:] == -128).all()
        assert np.array_equal(r["U"][b], d["U_init"][b])
        assert np.array_equal(r["X"][b], o["X"][b], equal_nan=True)
    assert r["status"][3] & 2 and np.isnan(r["best_cost"][3])
    assert not (r["status"][7] & 2) and np.isinf(r["best_cost"][7])


def test_bound_solve_equals_eager_calls():
    """BoundSolve (prepared arguments, bound outputs) returns what the eager
    entry points return, call after call with changing inputs."""
    d = load("cfg1_b16_t5")
    kw = case_kwargs(d)
    bs = nat.BoundSolve(16, 5, DEV, g(kw["u_min"]), g(kw["u_max"]), dt=kw["dt"], max_iter=kw["max_iter"],
                        reg_eps=kw["reg"], alphas=kw["alphas"])
    for scale in (1.0, 0.5):
        x0 = g(d["x0"] * np.float32(scale))
        out, grads = bs(x0, g(d["U_init"]), g(d["C"]), g(d["c"]), g(d["gX"]), g(d["gU"]))
        ref = nat.solve(x0, g(d["U_init"]), g(d["C"]), g(d["c"]), None, None, None, None, g(kw["u_min"]),
                        g(kw["u_max"]), dt=kw["dt"], max_iter=kw["max_iter"], reg_eps=kw["reg"], alphas=kw["alphas"])
        rg = nat.backward(ref["X"], ref["U"], g(d["C"]), g(d["gX"]), g(d["gU"]), tight=ref["tight"], dt=kw["dt"],
                          reg_eps=kw["reg"])
        for k in ("X", "U", "tight"):
            assert torch.equal(out[k], ref[k]), k
        for k in ("x0", "C", "c"):
            assert torch.equal(grads[k], rg[k]), k
    with pytest.raises(RuntimeError, match="float32"):
        bs(g(d["x0"]).double(), g(d["U_init"]), g(d["C"]), g(d["c"]))


def test_empty_batch():
    z = lambda *s: torch.zeros(*s, device=DEV)
    out = nat.solve(z(0, 10), z(0, 3, 4), z(0, 3, 14, 14), z(0, 3, 14))
    assert out["X"].shape == (0, 4, 10)


def sample_indices(B, n=512, tail=8):
    """A strided sample of n elements of a batch of B that touches every
    1024-element block, lands at varying positions inside warps, and includes
    the last `tail` elements (the ragged last warp)."""
    stride = max(1, B // n)
    j = np.arange(n)
    idx = j * stride + (7 * j) % stride
    return np.unique(np.concatenate([idx[idx < B], np.arange(max(0, B - tail), B)]))


def replay_sample(cfg, inp, res, grads, gX, gU, idx):
    """The oracle replays the GPU's own decisions on the sampled elements: X, U
    within 1e-4 of the GPU's, and the oracle's backward at the GPU's solution
    within 1e-3 of the GPU's gradients, per element. Two fp32 implementations
    with different summation orders can only agree as far as the problem's
    conditioning allows, so the bar is per element the plain one or
    CONDITION_FACTOR times the oracle's response to 1e-7 noise in C (about one
    ulp), whichever is larger, where that response times CONDITION_FACTOR
    stays below 0.05; the rest (one ulp moves them further; long horizons
    have such elements) are compared with the oracle's fp64 replay instead,
    within 30 times the oracle's own fp32 error."""
    from parity import CONDITION_FACTOR, condition_spread, rel_per_elem
    sl = {k: np.ascontiguousarray(v[idx]) for k, v in inp.items()}
    tr = res["trace"][idx].cpu().numpy()
    X, U = res["X"][idx].cpu().numpy(), res["U"][idx].cpu().numpy()
    tight = res["tight"][idx].cpu().numpy()
    kw = dict(u_min=wl.U_MIN, u_max=wl.U_MAX, dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"], forced=tr)

    def run(C):
        o_ = O.solve(sl["x0"], sl["U_init"], C, sl["c"], **kw)
        out = {"X": o_["X"], "U": o_["U"]}
        if grads is not None:
            g_ = O.backward(X, U, C, None, None, None, tight, gX[idx], gU[idx], wl.DT, wl.REG_EPS)
            out.update({k: g_["grad_" + k] for k in grads})
        return out

    o = run(sl["C"])
    gpu = {"X": X, "U": U}
    if grads is not None:
        gpu.update({k: grads[k][idx].cpu().numpy() for k in grads})
    sp = condition_spread(run, sl["C"], rel_per_elem)
    ill = np.zeros(len(idx), bool)
    for k in gpu:
        ill |= CONDITION_FACTOR * sp[k] > 0.05
    for k in gpu:
        tol = TOL_XU if k in ("X", "U") else TOL_GRAD
        err = rel_per_elem(gpu[k], o[k])
        bad = np.nonzero(~ill & (err > np.maximum(tol, CONDITION_FACTOR * sp[k])))[0]
        assert bad.size == 0, (k, [(int(idx[b]), float(err[b]), float(sp[k][b])) for b in bad])
    if ill.any():
        o64 = O.solve(sl["x0"], sl["U_init"], sl["C"], sl["c"], dtype=np.float64, **kw)
        for k in ("X", "U"):
            e_gpu, e_o32 = rel_per_elem(gpu[k], o64[k]), rel_per_elem(o[k], o64[k])
            bad = np.nonzero(ill & (e_gpu > np.maximum(TOL_XU, 30.0 * e_o32)))[0]
            assert bad.size == 0, (k, [(int(idx[b]), float(e_gpu[b]), float(e_o32[b])) for b in bad])


@pytest.mark.parametrize("B,T,iters", [(16384, 20, 5)])
def test_training_scale_properties(B, T, iters):
    """Full training-scale batch: deterministic, finite, its first 16 elements
    equal the 16-element solve (which the replay tests pin to the reference),
    the backward is exactly linear in the upstream gradient (x2 scaling), and
    a strided sample of 520 elements (every 1024-block, the ragged last warp)
    is replayed by the oracle from the GPU's own decisions: X, U within 1e-4
    and the gradients within 1e-3, or the element's conditioning bar
    (replay_sample)."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=B)
    t = {k: g(v) for k, v in inp.items()}
    args = (t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, g(wl.U_MIN), g(wl.U_MAX))
    kw = dict(dt=wl.DT, max_iter=iters, alphas=cfg["alphas"], want_trace=True)
    a = nat.solve(*args, **kw)
    b = nat.solve(*args, **kw)
    assert torch.equal(a["X"], b["X"]) and torch.equal(a["U"], b["U"])
    assert torch.isfinite(a["X"]).all() and torch.isfinite(a["U"]).all()
    small = load("cfg3_b16_t20")
    r16, _ = gpu_solve(small)
    assert np.array_equal(a["X"][:16].cpu().numpy(), r16["X"])
    gX, gU = wl.make_backward_seeds(B, T)
    g1 = nat.backward(a["X"], a["U"], t["C"], g(gX), g(gU), tight=a["tight"], dt=wl.DT)
    g2 = nat.backward(a["X"], a["U"], t["C"], g(2 * gX), g(2 * gU), tight=a["tight"], dt=wl.DT)
    for k in g1:
        assert torch.equal(2 * g1[k], g2[k]), k
    replay_sample(cfg, inp, a, g1, gX, gU, sample_indices(B))


@pytest.mark.parametrize("layout", ["team", "pair"])
def test_diag_cost_cache_identical_to_dense_path(monkeypatch, layout):
    """Diagonal C blocks are detected in the first pass and later passes read
    only their diagonals. Every result must equal the dense path's
    (ILQR_B200_DIAG_CACHE=0): here with one warp (six elements in the team
    layout, two in the pair layout) holding a single off-diagonal entry (that
    warp stays dense) and one element that starts at an infinite position (the
    quadratic form's 0 * inf = NaN rule)."""
    monkeypatch.setenv("ILQR_B200_LAYOUT", layout)
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=96)
    inp["C"][7, 3, 2, 5] = inp["C"][7, 3, 5, 2] = np.float32(1e-3)
    inp["x0"][20, 0] = np.inf
    t = {k: g(v) for k, v in inp.items()}
    args = (t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, g(wl.U_MIN), g(wl.U_MAX))
    kw = dict(dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"], want_trace=True, want_stats=True)
    on = {k: v.cpu().numpy() for k, v in nat.solve(*args, **kw).items()}
    monkeypatch.setenv("ILQR_B200_DIAG_CACHE", "0")
    off = {k: v.cpu().numpy() for k, v in nat.solve(*args, **kw).items()}
    diag_bit = 8
    assert not (off["status"] & diag_bit).any()
    warp_dense = np.zeros(96, bool)
    warp_dense[6:12 if layout == "team" else 8] = True
    assert ((on["status"] & diag_bit) != 0).tolist() == (~warp_dense).tolist()
    assert not np.isfinite(off["X"][20]).all()
    for k in on:
        a, b = on[k], off[k]
        if k == "status":
            a = a & ~diag_bit
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k


@pytest.mark.parametrize("forced", [False, True])
def test_more_step_sizes_than_candidate_slots(forced):
    """Seven step sizes: the first five candidates are kept in workspace slots,
    the last two are re-run when accepted. Free-running and replaying a trace
    that accepts step sizes 6 and 7, the GPU matches the oracle given the same
    decisions."""
    d = dict(load("cfg3_b16_t20"))
    d["alphas"] = np.array([1.0, 0.8, 0.6, 0.5, 0.3, 0.2, 0.1], np.float32)
    trace = None
    if forced:
        trace = np.tile(np.array([[5, 6, 0, -1, 6, 2, 5, -1, -1, 4]], np.int8), (16, 1))
        trace = trace[:, : int(d["max_iter"])]
        trace[1::3] = np.roll(trace[1::3], 2, axis=1)
    r, kw = gpu_solve(d, forced=trace)
    o = O.solve(d["x0"], d["U_init"], d["C"], d["c"], forced=r["trace"] if trace is None else trace, **kw)
    assert max_rel(r["X"], o["X"]) <= TOL_XU
    assert max_rel(r["U"], o["U"]) <= TOL_XU
    if forced:
        acc = trace >= 0
        assert (r["trace"][acc] == trace[acc]).all()


def _sig_spec(d):
    return nat.SigmoidCostSpec(float(d["cost_eps"]), float(d["range_q"]), float(d["range_p"]),
                               range_pt=float(d["range_pt"]))


def test_sigmoid_cost_replay_matches_reference():
    """Costs built in the kernel from the policy's sigmoid output: replaying the
    reference's decisions, X, U match within 1e-4 and the gradient of the
    sigmoid output within 1e-3 (reference: _build_cost_tensors + DiffMPC +
    autograd)."""
    d = load("sigmoid_b16_t10")
    kw = case_kwargs(d)
    spec = _sig_spec(d)
    r = nat.solve_sigmoid(g(d["x0"]), g(d["U_init"]), g(d["sigmoid_cost"]), spec, g(kw["u_min"]),
                          g(kw["u_max"]), dt=kw["dt"], max_iter=kw["max_iter"], reg_eps=kw["reg"],
                          alphas=kw["alphas"], forced_trace=g(d["ref_trace"], torch.int8))
    assert max_rel(r["X"].cpu().numpy(), d["ref_X"]) <= TOL_XU
    assert max_rel(r["U"].cpu().numpy(), d["ref_U"]) <= TOL_XU
    assert np.array_equal(r["tight"].cpu().numpy().astype(bool), d["ref_tight"])
    gr = nat.backward_sigmoid(g(d["ref_X"]), g(d["ref_U"]), g(d["sigmoid_cost"]), g(d["gX"]), g(d["gU"]),
                              spec, tight=g(d["ref_tight"], torch.uint8), dt=kw["dt"], reg_eps=kw["reg"])
    assert max_rel(gr["sigmoid_cost"].cpu().numpy(), d["ref_grad_sigmoid_cost"]) <= TOL_GRAD
    assert max_rel(gr["x0"].cpu().numpy(), d["ref_grad_x0"]) <= TOL_GRAD


def test_sigmoid_cost_path_equals_dense_path():
    """On the dense C, c the policy would build from the same sigmoid output,
    the dense entry points give bit-identical solves, and their gradients
    chained through the construction equal the sigmoid backward's, at
    B=600, T=20 (free-running decisions included)."""
    B, T = 600, 20
    rng = np.random.default_rng(8)
    sc = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.5, (B, 28 * T))))).astype(np.float32)
    inp = wl.make_inputs(B, T, seed=2)
    spec = nat.SigmoidCostSpec()
    C, c = O.sigmoid_costs(sc, T, *spec.args())
    common = dict(dt=wl.DT, max_iter=5, alphas=(1.0, 0.8, 0.5, 0.2, 0.1), want_trace=True, want_stats=True)
    x0, Ui, lo, hi = g(inp["x0"]), g(inp["U_init"]), g(wl.U_MIN), g(wl.U_MAX)
    dn = nat.solve(x0, Ui, g(C), g(c), None, None, None, None, lo, hi, **common)
    sg = nat.solve_sigmoid(x0, Ui, g(sc), spec, lo, hi, **common)
    for k in dn:
        a, b = dn[k].cpu().numpy(), sg[k].cpu().numpy()
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k
    gX, gU = (g(a) for a in wl.make_backward_seeds(B, T))
    gd = nat.backward(dn["X"], dn["U"], g(C), gX, gU, tight=dn["tight"], dt=wl.DT, need=("x0", "C", "c"))
    gs = nat.backward_sigmoid(sg["X"], sg["U"], g(sc), gX, gU, spec, tight=sg["tight"], dt=wl.DT)
    chained = O.sigmoid_cost_grad(gd["C"].cpu().numpy(), gd["c"].cpu().numpy(), T, spec.range_q,
                                  spec.range_p, spec.range_pt)
    assert np.array_equal(chained, gs["sigmoid_cost"].cpu().numpy())
    assert torch.equal(gd["x0"], gs["x0"])


def test_fastmpc_sigmoid_cost_autograd():
    """FastMPC with a SigmoidQuadCost: the same X, U as a QuadCost of the
    policy's dense costs, and autograd delivers the kernel's gradient of the
    sigmoid output."""
    d = load("sigmoid_b16_t10")
    T = d["U_init"].shape[1]
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    mpc = mpc_compat.FastMPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                             u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=int(d["max_iter"]),
                             eps=1e-6)
    x0 = g(d["x0"])
    sc = g(d["sigmoid_cost"]).requires_grad_(True)
    x, u, _ = mpc(x0, mpc_compat.SigmoidQuadCost(sc), _dx())
    C = g(d["C"]).permute(1, 0, 2, 3)
    c = g(d["c"]).permute(1, 0, 2)
    with torch.no_grad():
        xd, ud, _ = mpc(x0, mpc_compat.QuadCost(C, c), _dx())
    assert torch.equal(x, xd) and torch.equal(u, ud)
    gx, gu = g(d["gX"]).permute(1, 0, 2), g(d["gU"]).permute(1, 0, 2)
    ((x * gx).sum() + (u * gu).sum()).backward()
    spec = nat.SigmoidCostSpec()
    out = nat.solve_sigmoid(x0, g(d["U_init"]), g(d["sigmoid_cost"]), spec, lo, hi, dt=wl.DT,
                            max_iter=int(d["max_iter"]), reg_eps=1e-6)
    ref = nat.backward_sigmoid(out["X"], out["U"], g(d["sigmoid_cost"]), g(d["gX"]), g(d["gU"]), spec,
                               tight=out["tight"], dt=wl.DT, reg_eps=1e-6)
    assert torch.equal(sc.grad, ref["sigmoid_cost"])


@pytest.mark.parametrize("sigmoid", [False, True])
def test_captured_solve_equals_eager_calls(sigmoid):
    """A solve + backward captured in a CUDA graph and replayed with new inputs
    gives the eager entry points' results bit for bit."""
    B, T, iters = 40, 8, 4
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    spec = nat.SigmoidCostSpec() if sigmoid else None
    cap = nat.CapturedSolve(B, T, DEV, lo, hi, dt=wl.DT, max_iter=iters, spec=spec)
    rng = np.random.default_rng(9)
    for seed in (1, 2):
        inp = wl.make_inputs(B, T, seed=seed)
        gX, gU = (g(a) for a in wl.make_backward_seeds(B, T, seed=seed))
        x0, Ui = g(inp["x0"]), g(inp["U_init"])
        if sigmoid:
            sc = g((1 / (1 + np.exp(-rng.normal(0, 1.5, (B, 28 * T))))).astype(np.float32))
            out, gr = cap(x0, Ui, grad_X=gX, grad_U=gU, sigmoid_cost=sc)
            ref = nat.solve_sigmoid(x0, Ui, sc, spec, lo, hi, dt=wl.DT, max_iter=iters)
            rg = nat.backward_sigmoid(ref["X"], ref["U"], sc, gX, gU, spec, tight=ref["tight"], dt=wl.DT)
        else:
            C, c = g(inp["C"]), g(inp["c"])
            out, gr = cap(x0, Ui, C, c, gX, gU)
            ref = nat.solve(x0, Ui, C, c, None, None, None, None, lo, hi, dt=wl.DT, max_iter=iters)
            rg = nat.backward(ref["X"], ref["U"], C, gX, gU, tight=ref["tight"], dt=wl.DT)
        torch.cuda.synchronize()
        for k in ("X", "U", "tight"):
            assert torch.equal(out[k], ref[k]), (seed, k)
        for k in rg:
            assert torch.equal(gr[k], rg[k]), (seed, k)


@pytest.mark.parametrize("name", ["inference_b262144_t10", "stress_b65536_t50"])
def test_full_size_configs(name):
    """The largest configurations run at full size (many waves of CTAs, 2-3 GB
    of costs): finite results, the first 16 elements equal to a 16-element
    solve of the same inputs, for the stress case a backward that is linear
    in the upstream gradient, and a strided sample of about 520 elements
    replayed by the oracle from the GPU's own decisions (replay_sample)."""
    cfg, inp = wl.config_inputs(name)
    B, T = cfg["B"], cfg["T"]
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    t = {k: g(v) for k, v in inp.items()}
    kw = dict(dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"])
    a = nat.solve(t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, lo, hi, want_trace=True, **kw)
    assert torch.isfinite(a["X"]).all() and torch.isfinite(a["U"]).all()
    s = nat.solve(*(t[k][:16].contiguous() for k in ("x0", "U_init", "C", "c")), None, None, None, None,
                  lo, hi, **kw)
    assert torch.equal(a["X"][:16], s["X"]) and torch.equal(a["U"][:16], s["U"])
    g1 = gX = gU = None
    if cfg["backward"]:
        gX, gU = wl.make_backward_seeds(B, T)
        g1 = nat.backward(a["X"], a["U"], t["C"], g(gX), g(gU), tight=a["tight"], dt=wl.DT, need=("x0", "c"))
        g2 = nat.backward(a["X"], a["U"], t["C"], g(2 * gX), g(2 * gU), tight=a["tight"], dt=wl.DT,
                          need=("x0", "c"))
        for k in g1:
            assert torch.isfinite(g1[k]).all()
            assert torch.equal(2 * g1[k], g2[k]), k
    del t
    replay_sample(cfg, inp, a, g1, gX, gU, sample_indices(B))


def test_pnqp4_batch_matches_oracle_and_optimum():
    """drone_pnqp4_batch on the GPU: the same iterates as the oracle's
    restatement (to fp32 rounding) and the exact box-QP optimum on all but a
    few hard problems; a warm start at the optimum stays there."""
    d = np.load(os.path.join(GOLDEN_DIR, "pnqp4_n256.npz"))
    ext = drone_ilqr.load_drone_ilqr_ext()
    H, q, lo, hi = (g(d[k]) for k in ("H", "q", "lower", "upper"))
    x, free = ext.drone_pnqp4_batch(H, q, lo, hi, None)
    x, free = x.cpu().numpy(), free.cpu().numpy()
    ox, ofree = O.pnqp4(d["H"], d["q"], d["lower"], d["upper"])
    scale = np.maximum(1.0, np.abs(ox).max(axis=1, keepdims=True))
    close = (np.abs(x - ox) / scale).max(axis=1) <= 1e-4
    assert close.sum() >= 250 and (free[close] == ofree[close]).all()
    at_opt = (np.abs(x - d["opt_x"]) / np.maximum(1.0, np.abs(d["opt_x"]).max(1, keepdims=True))).max(1) <= 1e-4
    assert at_opt.sum() >= 250
    assert (x >= d["lower"]).all() and (x <= d["upper"]).all()
    xw, fw = ext.drone_pnqp4_batch(H, q, lo, hi, g(d["opt_x"].astype(np.float32)))
    assert (np.abs(xw.cpu().numpy() - d["opt_x"]).max(1) <= 1e-4 * np.maximum(1.0, np.abs(d["opt_x"]).max(1))).sum() >= 250
