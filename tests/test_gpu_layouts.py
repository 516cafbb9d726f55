"""The two kernel layouts of the 10-state solve and backward give the same
bits: the team layout (six elements per warp, five lanes each) and the pair
layout (two elements per warp, sixteen lanes each; the default for small
batches). ILQR_B200_LAYOUT forces one layout; every output of the solve
(X, U, tight mask, decision trace, iterations, best cost, stall record, the
status bits other than the diagonal-cost flag, which depends on which
elements share a warp) and every gradient of the backward are compared bit
for bit, on the golden cases (dense and asymmetric costs with terminal cost
and references, no box, an indefinite Q_uu that takes the SVD fallback),
an odd training-scale batch, a non-finite element, seven step sizes with
re-run candidates, sigmoid costs and the time-major layout."""

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl
from parity import case_kwargs, load

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DIAG_BIT = 8
NEED = ("x0", "C", "c", "C_final", "c_final", "x_ref", "u_ref")


def g(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, dtype)


def _eq(a, b, key):
    a, b = a.cpu().numpy(), b.cpu().numpy()
    if key == "status":
        a, b = a & ~DIAG_BIT, b & ~DIAG_BIT
    assert a.shape == b.shape, key
    assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), key


def _both(monkeypatch, fn):
    out = {}
    for layout in ("team", "pair"):
        monkeypatch.setenv("ILQR_B200_LAYOUT", layout)
        out[layout] = fn()
        torch.cuda.synchronize()
    monkeypatch.delenv("ILQR_B200_LAYOUT")
    return out["team"], out["pair"]


def _solve_and_backward(d, kw, forced=None, time_major=False):
    C, c = g(d["C"]), g(d["c"])
    gX, gU = g(d["gX"]), g(d["gU"])
    if time_major:
        C, c = C.transpose(0, 1).contiguous(), c.transpose(0, 1).contiguous()
    s = nat.solve(g(d["x0"]), g(d["U_init"]), C, c, g(kw["C_f"]), g(kw["c_f"]), g(kw["x_ref"]), g(kw["u_ref"]),
                  g(kw["u_min"]), g(kw["u_max"]), dt=kw["dt"], max_iter=kw["max_iter"], reg_eps=kw["reg"],
                  alphas=kw["alphas"], forced_trace=g(forced, torch.int8), want_trace=True, want_stats=True,
                  time_major=time_major)
    r = nat.backward(s["X"], s["U"], C, gX, gU, C_final=g(kw["C_f"]), x_ref=g(kw["x_ref"]),
                     u_ref=g(kw["u_ref"]), tight=s["tight"], dt=kw["dt"], reg_eps=kw["reg"],
                     need=NEED if kw["C_f"] is not None or kw["x_ref"] is not None else ("x0", "C", "c"),
                     time_major=time_major)
    return s, r


def _check(a, b):
    (sa, ra), (sb, rb) = a, b
    assert set(sa) == set(sb)
    for k in sa:
        _eq(sa[k], sb[k], k)
    for k in ra:
        _eq(ra[k], rb[k], "grad_" + k)


@pytest.mark.parametrize("name", ["cfg1_b16_t5", "cfg3_b16_t20", "dense_b8_t6", "asym_b8_t4", "nobox_b8_t5",
                                  "indef_b8_t4", "b1_t1"])
def test_golden_cases_same_bits(monkeypatch, name):
    d = load(name)
    kw = case_kwargs(d)
    _check(*_both(monkeypatch, lambda: _solve_and_backward(d, kw)))


@pytest.mark.parametrize("time_major", [False, True])
def test_odd_training_batch_same_bits(monkeypatch, time_major):
    """B = 45 at the training-scale horizon: the last warp of either layout is
    ragged, and one element starts at an infinite position."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=45)
    inp["x0"][31, 0] = np.inf
    gX, gU = wl.make_backward_seeds(45, cfg["T"])
    d = dict(inp, gX=gX, gU=gU)
    kw = dict(C_f=None, c_f=None, x_ref=None, u_ref=None, u_min=wl.U_MIN, u_max=wl.U_MAX, dt=wl.DT,
              max_iter=cfg["max_iter"], reg=wl.REG_EPS, alphas=cfg["alphas"])
    team, pair = _both(monkeypatch, lambda: _solve_and_backward(d, kw, time_major=time_major))
    _check(team, pair)
    assert not np.isfinite(pair[0]["X"][31].cpu().numpy()).all()


@pytest.mark.parametrize("forced", [False, True])
def test_seven_step_sizes_same_bits(monkeypatch, forced):
    d = dict(load("cfg3_b16_t20"))
    kw = case_kwargs(d)
    kw["alphas"] = (1.0, 0.8, 0.6, 0.5, 0.3, 0.2, 0.1)
    trace = None
    if forced:
        trace = np.tile(np.array([[5, 6, 0, -1, 6]], np.int8), (16, 1))[:, : kw["max_iter"]]
    _check(*_both(monkeypatch, lambda: _solve_and_backward(d, kw, forced=trace)))


def test_sigmoid_costs_same_bits(monkeypatch):
    d = load("sigmoid_b16_t10")
    spec = nat.SigmoidCostSpec(float(d["cost_eps"]), float(d["range_q"]), float(d["range_p"]),
                               range_pt=float(d["range_pt"]))
    sc = g(d["sigmoid_cost"])
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)

    def run():
        s = nat.solve_sigmoid(g(d["x0"]), g(d["U_init"]), sc, spec, lo, hi, dt=float(d["dt"]),
                              max_iter=int(d["max_iter"]), reg_eps=float(d["reg"]),
                              alphas=tuple(float(a) for a in d["alphas"]), want_trace=True, want_stats=True)
        r = nat.backward_sigmoid(s["X"], s["U"], sc, g(d["gX"]), g(d["gU"]), spec, tight=s["tight"],
                                 dt=float(d["dt"]), reg_eps=float(d["reg"]))
        return s, r

    _check(*_both(monkeypatch, run))


def test_default_layout_by_batch(monkeypatch):
    """The default picks the pair layout up to PAIR_MAX_B and the team layout
    above; the first elements of a batch just above the limit equal those of
    a batch just below it (prefix independence across the two layouts)."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=4100)
    t = {k: g(v) for k, v in inp.items()}
    kw = dict(dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"], want_trace=True)
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    big = nat.solve(t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, lo, hi, **kw)
    small = nat.solve(*(t[k][:4096].contiguous() for k in ("x0", "U_init", "C", "c")), None, None, None, None,
                      lo, hi, **kw)
    for k in ("X", "U", "tight", "trace"):
        assert torch.equal(big[k][:4096], small[k]), k


def _segmented_vs_whole(monkeypatch, inp, cfg, T):
    """Solve (and backward) with the segmented team solve and in one launch."""
    t = {k: g(v) for k, v in inp.items()}
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    gX, gU = (g(a) for a in wl.make_backward_seeds(t["x0"].shape[0], T))
    out = {}
    for seg in ("1", "0"):
        monkeypatch.setenv("ILQR_B200_SEGMENT", seg)
        s = nat.solve(t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, lo, hi, dt=wl.DT,
                      max_iter=cfg["max_iter"], alphas=cfg["alphas"], want_trace=True, want_stats=True)
        r = nat.backward(s["X"], s["U"], t["C"], gX, gU, tight=s["tight"], dt=wl.DT, reg_eps=wl.REG_EPS)
        torch.cuda.synchronize()
        out[seg] = (s, r)
    monkeypatch.delenv("ILQR_B200_SEGMENT")
    return out["1"], out["0"]


def test_segmented_team_solve_same_bits(monkeypatch):
    """Large team-layout batches run in two launches: every element for
    max_iter - 2 iterations, then the elements still improving, compacted six
    per warp. The training-scale batch (B = 16384, T = 20, 5 iterations, the
    diagonal costs the policy builds) gives the same bits as one launch: X, U,
    tight mask, trace, iterations, status, best cost, stall record and every
    gradient of the backward at the solution."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20")
    (s1, r1), (s0, r0) = _segmented_vs_whole(monkeypatch, inp, cfg, cfg["T"])
    assert int((s0["iters"] > cfg["max_iter"] - 2).sum()) > 1000  # the resumed launch has work
    for k in ("X", "U", "tight", "trace", "iters", "status", "best_cost", "stall_iter", "stall_gap"):
        a, b = s1[k].cpu().numpy(), s0[k].cpu().numpy()
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k
    for k in r0:
        assert torch.equal(r1[k], r0[k]), k


def test_segmented_team_solve_mixed_warps(monkeypatch):
    """A batch in which some warps hold a dense (non-diagonal) cost block: those
    warps finish in the first launch, the others resume; same bits as one
    launch."""
    cfg, inp = wl.config_inputs("rollout_b16384_t20", B=9000)
    C = inp["C"].copy()
    rng = np.random.default_rng(3)
    for b in rng.choice(9000, size=40, replace=False):  # one off-diagonal pair in some element's step
        t = int(rng.integers(0, cfg["T"]))
        C[b, t, 0, 1] = C[b, t, 1, 0] = 1e-3
    inp = dict(inp, C=C)
    (s1, r1), (s0, r0) = _segmented_vs_whole(monkeypatch, inp, cfg, cfg["T"])
    assert int(((s0["status"] & DIAG_BIT) == 0).sum()) > 0  # some warps dense
    for k in ("X", "U", "tight", "trace", "iters", "status", "best_cost", "stall_iter", "stall_gap"):
        a, b = s1[k].cpu().numpy(), s0[k].cpu().numpy()
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k
    for k in r0:
        assert torch.equal(r1[k], r0[k]), k


def test_segmented_team_solve_chain(monkeypatch):
    """More than five iterations run as a chain of launches, one per iteration
    after the first, each on the elements still improving (the long-horizon
    configuration: T = 50, 8 iterations, step sizes 1 .. 1/8, targets 15 m
    away); same bits as one launch."""
    cfg, inp = wl.config_inputs("stress_b65536_t50", B=8192)
    t = {k: g(v) for k, v in inp.items()}
    lo, hi = g(wl.U_MIN), g(wl.U_MAX)
    gX, gU = (g(a) for a in wl.make_backward_seeds(8192, cfg["T"]))
    out = {}
    for seg in ("1", "0"):
        monkeypatch.setenv("ILQR_B200_SEGMENT", seg)
        s = nat.solve(t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, lo, hi, dt=wl.DT,
                      max_iter=cfg["max_iter"], alphas=cfg["alphas"], want_trace=True, want_stats=True)
        r = nat.backward(s["X"], s["U"], t["C"], gX, gU, tight=s["tight"], dt=wl.DT, reg_eps=wl.REG_EPS)
        torch.cuda.synchronize()
        out[seg] = (s, r)
    monkeypatch.delenv("ILQR_B200_SEGMENT")
    (s1, r1), (s0, r0) = out["1"], out["0"]
    assert int((s0["iters"] > 2).sum()) > 100  # several launches of the chain have work
    for k in ("X", "U", "tight", "trace", "iters", "status", "best_cost", "stall_iter", "stall_gap"):
        a, b = s1[k].cpu().numpy(), s0[k].cpu().numpy()
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k
    for k in r0:
        assert torch.equal(r1[k], r0[k]), k


def test_segmented_team_solve_sigmoid_costs(monkeypatch):
    """Costs built in the kernel from the policy's sigmoid output take the
    segmented path too (diagonal from the start; the first launch keeps the cost
    records the resumed one reads); same bits as one launch, B = 9000, T = 20."""
    B, T = 9000, 20
    rng = np.random.default_rng(11)
    sc = g((1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.5, (B, 28 * T))))).astype(np.float32))
    inp = wl.make_inputs(B, T, seed=4)
    x0, Ui, lo, hi = g(inp["x0"]), g(inp["U_init"]), g(wl.U_MIN), g(wl.U_MAX)
    spec = nat.SigmoidCostSpec()
    out = {}
    for seg in ("1", "0"):
        monkeypatch.setenv("ILQR_B200_SEGMENT", seg)
        out[seg] = nat.solve_sigmoid(x0, Ui, sc, spec, lo, hi, dt=wl.DT, max_iter=5,
                                     alphas=(1.0, 0.8, 0.5, 0.2, 0.1), want_trace=True, want_stats=True)
        torch.cuda.synchronize()
    monkeypatch.delenv("ILQR_B200_SEGMENT")
    assert int((out["0"]["iters"] > 3).sum()) > 100
    for k in out["0"]:
        a, b = out["1"][k].cpu().numpy(), out["0"][k].cpu().numpy()
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), k
