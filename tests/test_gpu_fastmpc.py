"""GPU parity of the FastMPC numerics mode (ilqr_fastmpc.cu) against its
oracle (oracle/fastmpc_oracle.py).

The GPU records its line-search decisions and the iteration at which the
batch stopped; the oracle replays them (the decisions are rounding-level
ties in any fp32 implementation) and the remaining arithmetic must agree to
1e-4 on X, U (relative to the largest magnitude of the element) and 1e-3 on
the gradients. The kernels and the oracle share operation order; they differ
by the kernels' fused multiply-adds in matrix products, their approximate
(2-ulp) division, as in the reference's fast-math build, and by sinf, cosf
(CUDA's, within 2 ulp, against the host's).
"""

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl
import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
LO = np.array([0.0, -10.0, -10.0, -4.0], np.float32)
HI = np.array([34.0, 10.0, 10.0, 4.0], np.float32)
TOL_XU = 1e-4
TOL_GRAD = 1e-3


def _t(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, dtype)


def _case(name):
    """(inputs dict, options dict) of a named case."""
    if name == "cfg1_b16_t5":
        d = wl.make_inputs(16, 5, seed=0)
        return d, dict(u_min=LO, u_max=HI, max_iter=10, dt=0.05)
    if name == "cfg2_b64_t10":
        d = wl.make_inputs(64, 10, seed=1)
        return d, dict(u_min=LO, u_max=HI, max_iter=10, dt=0.05)
    if name == "cfg3_b48_t20":
        d = wl.make_inputs(48, 20, seed=2)
        return d, dict(u_min=LO, u_max=HI, max_iter=5, dt=0.05)
    if name == "dense_b8_t6":
        d = wl.make_inputs(8, 6, seed=3)
        extra = wl.make_dense_costs(8, 6, seed=4)
        d = dict(d, C=extra["C"], c=extra["c"])
        return d, dict(u_min=LO, u_max=HI, max_iter=6, dt=0.05, C_f=extra["C_final"], c_f=extra["c_final"],
                       x_ref=extra["x_ref"], u_ref=extra["u_ref"])
    if name == "nobox_b8_t5":
        d = wl.make_inputs(8, 5, seed=5)
        return d, dict(u_min=None, u_max=None, max_iter=5, dt=0.05)
    if name == "ragged_b13_t7":
        d = wl.make_inputs(13, 7, seed=6, r=15.0)
        return d, dict(u_min=LO, u_max=HI, max_iter=9, dt=0.05)
    if name == "cfg5_b8_t50":
        d = wl.make_inputs(8, 50, seed=7, r=15.0)
        return d, dict(u_min=LO, u_max=HI, max_iter=8, dt=0.05)
    raise KeyError(name)


# cfg5_b8_t50 (long horizon) is checked against the problem's conditioning instead
CASES = ["cfg1_b16_t5", "cfg2_b64_t10", "cfg3_b48_t20", "dense_b8_t6", "nobox_b8_t5", "ragged_b13_t7"]


def _gpu(d, o, time_major=False):
    tm = (lambda a: a.transpose(0, 1).contiguous()) if time_major else (lambda a: a)
    return nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), tm(_t(d["C"])), tm(_t(d["c"])), C_final=_t(o.get("C_f")),
                             c_final=_t(o.get("c_f")), x_ref=_t(o.get("x_ref")), u_ref=_t(o.get("u_ref")),
                             u_min=_t(o["u_min"]), u_max=_t(o["u_max"]), dt=o["dt"], max_iter=o["max_iter"],
                             want_trace=True, time_major=time_major)


def _np(out):
    return {k: v.cpu().numpy() for k, v in out.items()}


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    ax = tuple(range(1, a.ndim))
    scale = np.maximum(np.abs(b).max(axis=ax, keepdims=True), 1.0)
    return (np.abs(a - b) / scale).max(axis=ax)


def _oracle_replay(d, o, g):
    return O.fm_solve(d["x0"], d["U_init"], d["C"], d["c"], C_f=o.get("C_f"), c_f=o.get("c_f"),
                      x_ref=o.get("x_ref"), u_ref=o.get("u_ref"), u_min=o["u_min"], u_max=o["u_max"], dt=o["dt"],
                      max_iter=o["max_iter"], forced=g["trace"].astype(np.int64),
                      forced_stop=int(g["batch_info"][1]))


@pytest.mark.parametrize("name", CASES)
def test_fastmpc_replay_matches_oracle(name):
    d, o = _case(name)
    g = _np(_gpu(d, o))
    r = _oracle_replay(d, o, g)
    assert r["iters_run"] == g["batch_info"][1]
    for k in ("X", "U", "X_lin", "U_lin"):
        err = _rel(g[k], r[k])
        assert err.max() <= TOL_XU, (k, float(err.max()), int(err.argmax()))
    # the box QP's active sets: equal but for rare rounding-level flips of a
    # control that sits at its bound
    if o["u_min"] is not None:
        diff = g["tight"].astype(bool) != r["tight"]
        assert diff.mean() < 0.01, diff.mean()
    else:
        assert not g["tight"].any()
    # decisions run by the GPU are recorded for every iteration it ran
    run = g["trace"] != O.NOT_RUN
    assert (run.sum(axis=1) == g["batch_info"][1]).all()


@pytest.mark.parametrize("name", ["cfg1_b16_t5", "cfg3_b48_t20", "dense_b8_t6", "nobox_b8_t5"])
def test_fastmpc_backward_matches_oracle(name):
    d, o = _case(name)
    sol = _gpu(d, o)
    g = _np(sol)
    B, T = d["U_init"].shape[:2]
    gX, gU = wl.make_backward_seeds(B, T)
    need = ("x0", "C", "c", "C_final", "c_final", "x_ref", "u_ref")
    gg = nat.fastmpc_backward(sol["X"], sol["U"], sol["X_lin"], sol["U_lin"], _t(d["C"]), _t(gX), _t(gU),
                              tight=sol["tight"] if o["u_min"] is not None else None, C_final=_t(o.get("C_f")),
                              x_ref=_t(o.get("x_ref")), u_ref=_t(o.get("u_ref")), dt=o["dt"], need=need)
    r = O.fm_backward(g["X"], g["U"], g["X_lin"], g["U_lin"], d["C"], gX, gU,
                      g["tight"].astype(bool) if o["u_min"] is not None else None, C_f=o.get("C_f"),
                      x_ref=o.get("x_ref"), u_ref=o.get("u_ref"), dt=o["dt"])
    for k in need:
        got = gg[k].cpu().numpy()
        err = _rel(got, r[k])
        assert err.max() <= TOL_GRAD, (k, float(err.max()), int(err.argmax()))


def test_long_horizon_within_conditioning():
    """T = 50, targets at 15 m (28 % of controls tight), 8 iterations. With the
    decisions replayed, X and U agree with the oracle, and the gradients at each
    side's solution agree, to the plain bars or to CONDITION_FACTOR times the
    oracle's own response to 1e-7 noise in C, per element."""
    from parity import CONDITION_FACTOR, fm_condition_spread
    d, o = _case("cfg5_b8_t50")
    sol = _gpu(d, o)
    g = _np(sol)
    stop = int(g["batch_info"][1])
    r = _oracle_replay(d, o, g)
    B, T = d["U_init"].shape[:2]
    gX, gU = wl.make_backward_seeds(B, T)
    sp = fm_condition_spread(d, g["trace"].astype(np.int64), stop, o["u_min"], o["u_max"], o["dt"], o["max_iter"],
                             grad_seeds=(gX, gU))
    for k in ("X", "U"):
        err = _rel(g[k], r[k])
        bad = np.nonzero(err > np.maximum(TOL_XU, CONDITION_FACTOR * sp[k]))[0]
        assert bad.size == 0, (k, [(int(b), float(err[b]), float(sp[k][b])) for b in bad])
    gg = nat.fastmpc_backward(sol["X"], sol["U"], sol["X_lin"], sol["U_lin"], _t(d["C"]), _t(gX), _t(gU),
                              tight=sol["tight"], dt=o["dt"])
    rg = O.fm_backward(r["X"], r["U"], r["X_lin"], r["U_lin"], d["C"], gX, gU, r["tight"], dt=o["dt"])
    for k in ("x0", "C", "c"):
        err = _rel(gg[k].cpu().numpy(), rg[k])
        bad = np.nonzero(err > np.maximum(TOL_GRAD, CONDITION_FACTOR * sp[k]))[0]
        assert bad.size == 0, (k, [(int(b), float(err[b]), float(sp[k][b])) for b in bad])


def test_fastmpc_time_major_is_bit_identical():
    d, o = _case("dense_b8_t6")
    a = _gpu(d, o)
    b = _gpu(d, o, time_major=True)
    for k in ("X", "U", "tight", "X_lin", "U_lin", "trace", "best_cost", "batch_info"):
        assert torch.equal(a[k], b[k]), k
    B, T = d["U_init"].shape[:2]
    gX, gU = (_t(v) for v in wl.make_backward_seeds(B, T))
    C = _t(d["C"])
    ga = nat.fastmpc_backward(a["X"], a["U"], a["X_lin"], a["U_lin"], C, gX, gU, tight=a["tight"])
    gb = nat.fastmpc_backward(a["X"], a["U"], a["X_lin"], a["U_lin"], C.transpose(0, 1).contiguous(), gX, gU,
                              tight=a["tight"], time_major=True)
    assert torch.equal(ga["x0"], gb["x0"])
    assert torch.equal(ga["C"], gb["C"].transpose(0, 1))
    assert torch.equal(ga["c"], gb["c"].transpose(0, 1))


def test_fastmpc_no_iterations_and_single_step():
    d, o = _case("cfg1_b16_t5")
    o0 = dict(o, max_iter=0)
    g = _np(_gpu(d, o0))
    U0 = np.minimum(np.maximum(d["U_init"], LO), HI)
    assert np.array_equal(g["U"], U0)
    np.testing.assert_allclose(g["X"], O.fm_rollout(d["x0"], U0, o["dt"]), rtol=1e-5, atol=1e-5)
    assert not g["tight"].any() and g["batch_info"][1] == 0
    d1 = wl.make_inputs(5, 1, seed=9)
    g1 = _np(_gpu(d1, dict(o, max_iter=3)))
    r1 = _oracle_replay(d1, dict(o, max_iter=3), g1)
    assert _rel(g1["U"], r1["U"]).max() <= TOL_XU


def test_fastmpc_batch_stop_follows_tolerance():
    """The batch stops at the first check whose largest improvement is below
    the tolerance: a loose tolerance stops at iteration 4, a zero one never."""
    d, o = _case("cfg2_b64_t10")
    loose = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                              dt=0.05, max_iter=10, converge_tol=1e9, want_trace=True)
    info = loose["batch_info"].cpu().numpy()
    assert info[1] == 4 and info[0] == 1
    assert (loose["trace"][:, 4:].cpu().numpy() == O.NOT_RUN).all()
    never = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                              dt=0.05, max_iter=10, converge_tol=0.0)
    assert never["batch_info"].cpu().numpy()[1] == 10


def test_fastmpc_invalid_arguments():
    d, o = _case("cfg1_b16_t5")
    with pytest.raises(RuntimeError):
        nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=None)
    with pytest.raises(RuntimeError):
        nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), alphas=())


def test_fastmpc_operator_autograd_equals_entry_points():
    """MPC(..., numerics="fastmpc") hands QuadCost's [T,B,...] tensors to the
    time-major entry points; its outputs and autograd gradients equal the
    batch-major entry points' bit for bit."""
    import mpc_compat
    d, o = _case("cfg1_b16_t5")
    B, T = d["U_init"].shape[:2]
    lo = _t(LO).view(1, 1, 4).expand(T, B, 4)
    hi = _t(HI).view(1, 1, 4).expand(T, B, 4)
    m = mpc_compat.MPC(10, 4, T, u_lower=lo, u_upper=hi, u_init=_t(d["U_init"]).transpose(0, 1), lqr_iter=10,
                       numerics="fastmpc")
    x0 = _t(d["x0"]).requires_grad_(True)
    C = _t(d["C"]).transpose(0, 1).contiguous().requires_grad_(True)
    c = _t(d["c"]).transpose(0, 1).contiguous().requires_grad_(True)
    X, U, _ = m(x0, mpc_compat.QuadCost(C, c), type("Dx", (), {"dt": 0.05})())
    ref = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                            dt=0.05, max_iter=10)
    assert torch.equal(X.detach().transpose(0, 1), ref["X"])
    assert torch.equal(U.detach().transpose(0, 1), ref["U"])
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    ((X * gX.transpose(0, 1)).sum() + (U * gU.transpose(0, 1)).sum()).backward()
    g = nat.fastmpc_backward(ref["X"], ref["U"], ref["X_lin"], ref["U_lin"], _t(d["C"]), gX, gU, tight=ref["tight"],
                             dt=0.05)
    assert torch.equal(x0.grad, g["x0"])
    assert torch.equal(C.grad.transpose(0, 1), g["C"])
    assert torch.equal(c.grad.transpose(0, 1), g["c"])
    with torch.no_grad():
        Xi, Ui, _ = m(_t(d["x0"]), mpc_compat.QuadCost(C.detach(), c.detach()), type("Dx", (), {"dt": 0.05})())
    assert torch.equal(Xi, X.detach()) and torch.equal(Ui, U.detach())


def test_fastmpc_training_scale_prefix_identity():
    """At B = 16384, T = 20 every output is finite, and the first 512 elements
    equal a B = 512 solve bit for bit when both batches ran the same number of
    iterations (elements share nothing but the batch stop)."""
    B, T = 16384, 20
    d = wl.make_inputs(B, T, seed=11)
    full = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                             dt=0.05, max_iter=5, want_trace=True)
    part = nat.fastmpc_solve(_t(d["x0"][:512]), _t(d["U_init"][:512]), _t(d["C"][:512]), _t(d["c"][:512]),
                             u_min=_t(LO), u_max=_t(HI), dt=0.05, max_iter=5, want_trace=True)
    for k in ("X", "U", "X_lin", "U_lin", "best_cost"):
        assert torch.isfinite(full[k]).all(), k
    if int(full["batch_info"][1]) == int(part["batch_info"][1]):
        for k in ("X", "U", "X_lin", "U_lin", "tight", "trace", "best_cost"):
            assert torch.equal(full[k][:512], part[k]), k
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    g = nat.fastmpc_backward(full["X"], full["U"], full["X_lin"], full["U_lin"], _t(d["C"]), gX, gU,
                             tight=full["tight"])
    for k in ("x0", "C", "c"):
        assert torch.isfinite(g[k]).all(), k


def test_fastmpc_nonfinite_element_is_isolated():
    """A NaN in one element's costs gives that element a NaN cost: it never
    improves (U stays clamp(U_init), X its rollout), and its NaN improvement
    keeps the batch from stopping early, as the reference's batch-wide max does
    (drone_ilqr_ext.cpp:1029-1049). The other elements stay finite and match
    the oracle's replay."""
    d, o = _case("cfg2_b64_t10")
    d = dict(d, C=d["C"].copy())
    d["C"][3, 2, 0, 0] = np.nan
    g = _np(_gpu(d, o))
    assert g["batch_info"][1] == o["max_iter"] and g["batch_info"][0] == 0
    U0 = np.minimum(np.maximum(d["U_init"][3], LO), HI)
    assert np.array_equal(g["U"][3], U0)
    assert np.isfinite(g["X"][3]).all() and np.isnan(g["best_cost"][3])
    assert (g["trace"][3] < 0).all()
    others = np.arange(64) != 3
    assert np.isfinite(g["X"][others]).all() and np.isfinite(g["U"][others]).all()
    r = _oracle_replay(d, o, g)
    for k in ("X", "U"):
        assert _rel(g[k][others], r[k][others]).max() <= TOL_XU, k


@pytest.mark.parametrize("alphas", [(1.0,), (1.0, 0.7, 0.5, 0.3, 0.2, 0.1), (1.0, 0.9, 0.8, 0.6, 0.4, 0.3, 0.2, 0.1)])
def test_fastmpc_step_size_counts(alphas):
    """One step size, and more than four (two lanes per candidate instead of
    four): the replayed oracle agrees as for the reference grid."""
    d, o = _case("cfg2_b64_t10")
    g = _np(nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                              dt=0.05, max_iter=6, alphas=alphas, want_trace=True))
    r = O.fm_solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=LO, u_max=HI, dt=0.05, max_iter=6, alphas=alphas,
                   forced=g["trace"].astype(np.int64), forced_stop=int(g["batch_info"][1]))
    for k in ("X", "U", "X_lin", "U_lin"):
        assert _rel(g[k], r[k]).max() <= TOL_XU, k
    assert g["trace"].max() < len(alphas)


def test_fastmpc_operator_takes_sigmoid_costs():
    """MPC(..., numerics="fastmpc") with SigmoidQuadCost solves the dense costs
    the policy would build, and autograd returns their gradient carried back
    through the construction to the sigmoid output."""
    import mpc_compat
    B, T = 16, 5
    d = wl.make_inputs(B, T, seed=7)
    sc = np.random.default_rng(8).uniform(0.0, 1e-3, (B, 28 * T)).astype(np.float32)
    C, c = O.sigmoid_costs(sc, T)
    lo = _t(LO).view(1, 1, 4).expand(T, B, 4)
    hi = _t(HI).view(1, 1, 4).expand(T, B, 4)
    m = mpc_compat.MPC(10, 4, T, u_lower=lo, u_upper=hi, lqr_iter=6, numerics="fastmpc")
    dx = type("Dx", (), {"dt": 0.05})()
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    s = _t(sc).requires_grad_(True)
    X, U, _ = m(_t(d["x0"]), mpc_compat.SigmoidQuadCost(s), dx)
    ((X * gX.transpose(0, 1)).sum() + (U * gU.transpose(0, 1)).sum()).backward()
    Cd = _t(C).transpose(0, 1).contiguous().requires_grad_(True)
    cd = _t(c).transpose(0, 1).contiguous().requires_grad_(True)
    X2, U2, _ = m(_t(d["x0"]), mpc_compat.QuadCost(Cd, cd), dx)
    ((X2 * gX.transpose(0, 1)).sum() + (U2 * gU.transpose(0, 1)).sum()).backward()
    assert torch.equal(X, X2) and torch.equal(U, U2)
    want = O.sigmoid_cost_grad(Cd.grad.transpose(0, 1).cpu().numpy(), cd.grad.transpose(0, 1).cpu().numpy(), T)
    got = s.grad.cpu().numpy()
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6 * np.abs(want).max())
