"""GPU parity of the 13-state rotor-thrust solver (ilqr_dense.cu) against the
reference DiffMPC run on the same model (golden vectors from
tests/golden/make_rotor13_golden.py) and against the oracle.

On this model fp32 rounding is strongly amplified: the reference's own fp32
solution differs from its fp64 solution by up to O(1) on some elements at
T >= 10 (the fp32 Riccati recursion loses definiteness). The bars are
therefore the rounding-aware ones of parity.within_rounding: the plain bars
(1e-4 on X and U, 1e-3 on gradients) wherever the reference is
well-conditioned, and the reference's own fp32 scatter elsewhere.
"""

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl
import mpc_compat
import oracle as O
from parity import (GRAD_KEYS, R13_CASES, TOL_GRAD, TOL_XU, WELL_CONDITIONED, case_kwargs, load, max_rel,
                    rel_per_elem, rounding_spread, within_rounding)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, dtype)


def _np(out):
    return {k: v.cpu().numpy() for k, v in out.items()}


def _gpu_solve(d, forced=None, B=None, **over):
    kw = case_kwargs(d)
    kw.update(over)
    sl = slice(None) if B is None else slice(0, B)
    s = lambda a: None if a is None else a[sl]
    out = nat.rotor13_solve(
        _t(d["x0"][sl]), _t(d["U_init"][sl]), _t(d["C"][sl]), _t(d["c"][sl]), C_final=_t(s(kw["C_f"])),
        c_final=_t(s(kw["c_f"])), x_ref=_t(s(kw["x_ref"])), u_ref=_t(s(kw["u_ref"])), u_min=_t(kw["u_min"]),
        u_max=_t(kw["u_max"]), dt=kw["dt"], max_iter=kw["max_iter"], reg_eps=kw["reg"], alphas=kw["alphas"],
        forced_trace=None if forced is None else _t(forced[sl], torch.int8), want_trace=True, want_stats=True)
    return _np(out)


def _oracle(d, forced, dtype=np.float32, B=None, **over):
    kw = case_kwargs(d)
    kw.update(over)
    sl = slice(None) if B is None else slice(0, B)
    s = lambda a: None if a is None else a[sl]
    for k in ("C_f", "c_f", "x_ref", "u_ref"):
        kw[k] = s(kw[k])
    r = O.solve(d["x0"][sl], d["U_init"][sl], d["C"][sl], d["c"][sl], forced=forced[sl], model=O.ROTOR13,
                dtype=dtype, **kw)
    return r, kw


def _perturb(d, seed, keys=("x0", "U_init", "C", "c")):
    """A copy of the inputs with each entry moved by about 2 ulp (seeded
    signs): another fp32 realisation of the same problem."""
    rng = np.random.default_rng(seed)
    out = dict(d)
    for k in keys:
        a = np.asarray(d[k], np.float64)
        out[k] = (a * (1.0 + 2.0 ** -22 * rng.choice([-1.0, 1.0], size=a.shape))).astype(np.float32)
    return out


def _realisations(d, trace, B=None, **over):
    """(fp64 solution, [fp32 realisations]) of the oracle replaying `trace`:
    the inputs as given and two perturbed copies."""
    o64, _ = _oracle(d, trace, np.float64, B, **over)
    reals = [_oracle(d, trace, np.float32, B, **over)[0]]
    reals += [_oracle(_perturb(d, sd), trace, np.float32, B, **over)[0] for sd in (1, 2)]
    return o64, reals


def _check_rounding(mine, o64, reals, key, tol, ref32=None):
    """within_rounding with the spread of all fp32 realisations at hand."""
    cands = [r[key] for r in reals] + ([ref32] if ref32 is not None else [])
    # a realisation that is not finite where the fp64 one is: unbounded scatter
    spread = np.max([np.nan_to_num(rel_per_elem(c, o64[key]), nan=np.inf) for c in cands], axis=0)
    return within_rounding(mine, cands[-1] if ref32 is not None else reals[0][key], o64[key], spread, tol)


def _gpu_backward(d, X, U, tight, kw, B=None):
    sl = slice(None) if B is None else slice(0, B)
    s = lambda a: None if a is None else a[sl]
    g = nat.rotor13_backward(_t(X), _t(U), _t(d["C"][sl]), _t(d["gX"][sl]), _t(d["gU"][sl]),
                             C_final=_t(s(kw["C_f"])), x_ref=_t(s(kw["x_ref"])), u_ref=_t(s(kw["u_ref"])),
                             tight=_t(tight, torch.uint8), dt=kw["dt"], reg_eps=kw["reg"],
                             need=("x0", "C", "c", "C_final", "c_final", "x_ref", "u_ref"))
    g = _np(g)
    return {"grad_x0": g["x0"], "grad_C": g["C"], "grad_c": g["c"], "grad_C_final": g["C_final"],
            "grad_c_final": g["c_final"], "grad_xref": g["x_ref"], "grad_uref": g["u_ref"]}


def _oracle_backward(d, X, U, tight, kw, dtype=np.float32):
    return O.backward(X, U, d["C"][: len(X)], kw["C_f"], kw["x_ref"], kw["u_ref"], tight, d["gX"][: len(X)],
                      d["gU"][: len(X)], kw["dt"], kw["reg"], dtype=dtype, model=O.ROTOR13)


def test_rotor13_dynamics_and_jacobian_bit_exact():
    """The device step equals the torch f_dyn the reference ran and the
    numpy model bit for bit; the Jacobian equals the numpy model's bit for
    bit (and the reference's autodiff Jacobian to rounding)."""
    d = load("r13_dynamics_n64")
    dt = float(d["dt"])
    xn = nat.rotor13_dynamics(_t(d["x"]), _t(d["u"]), dt).cpu().numpy()
    assert np.array_equal(xn, d["x_next"])
    X = np.stack([d["x"], d["x_next"]], axis=1)
    A, Bm = nat.rotor13_linearize(_t(X), _t(d["u"][:, None, :]), dt)
    Ao, Bo = O.rotor13_jacobian(d["x"], d["u"], dt)
    assert np.array_equal(A.cpu().numpy()[:, 0], Ao)
    assert np.array_equal(Bm.cpu().numpy()[:, 0], Bo)


@pytest.mark.parametrize("name", R13_CASES)
def test_rotor13_replay_matches_reference(name):
    """With the reference's fp32 decisions replayed: X, U within the
    rounding-aware bars, the replayed trace reported back, the tight mask
    equal on well-conditioned elements."""
    d = load(name)
    r = _gpu_solve(d, forced=d["ref_trace"])
    # the replayed decisions come back; a rejection records the kernel's own argmin
    acc = d["ref_trace"] >= 0
    assert np.array_equal(r["trace"] >= 0, acc)
    assert np.array_equal(r["trace"][acc], d["ref_trace"][acc])
    assert np.array_equal(r["trace"] == -128, d["ref_trace"] == -128)
    o64, reals = _realisations(d, d["ref_trace"])
    for key in ("X", "U"):
        fails = _check_rounding(r[key], o64, reals, key, TOL_XU, ref32=d["ref_" + key])
        assert not fails, (key, fails)
    well = rounding_spread(d["ref_U"], reals[0]["U"], o64["U"]) <= WELL_CONDITIONED
    assert np.array_equal(r["tight"][well].astype(bool), d["ref_tight"][well])


@pytest.mark.parametrize("name", R13_CASES)
def test_rotor13_backward_at_reference_solution(name):
    """The implicit-diff backward alone, at the reference's (X, U, mask)."""
    d = load(name)
    kw = case_kwargs(d)
    X, U, tight = d["ref_X"], d["ref_U"], d["ref_tight"]
    g = _gpu_backward(d, X, U, tight.astype(np.uint8), kw)
    g64 = _oracle_backward(d, X, U, tight, kw, np.float64)
    reals = [_oracle_backward(d, X, U, tight, kw)]
    for sd in (1, 2):
        p = _perturb(dict(d, X=X, U=U), sd, keys=("X", "U", "C"))
        reals.append(_oracle_backward(p, p["X"], p["U"], tight, kw))
    for k in GRAD_KEYS:
        fails = _check_rounding(g[k], g64, reals, k, TOL_GRAD, ref32=d["ref_" + k])
        assert not fails, (k, fails)


@pytest.mark.parametrize("name", ["r13_cfg1_b16_t5", "r13_cfg3_b16_t20", "r13_dense_b8_t6"])
def test_rotor13_free_run_against_oracle_replay(name):
    """Free-running, the kernel's own decisions replayed in the oracle give
    the same X, U within the rounding-aware bars; every element's objective
    is no worse than the initial one."""
    d = load(name)
    r = _gpu_solve(d)
    kw = case_kwargs(d)
    o64, reals = _realisations(d, r["trace"])
    for key in ("X", "U"):
        fails = _check_rounding(r[key], o64, reals, key, TOL_XU)
        assert not fails, (key, fails)
    X0 = O.rollout(d["x0"], d["U_init"], kw["dt"], O.ROTOR13)
    B, T = d["U_init"].shape[:2]
    zx = np.zeros((B, T + 1, 13), np.float32) if kw["x_ref"] is None else kw["x_ref"]
    zu = np.zeros((B, T, 4), np.float32) if kw["u_ref"] is None else kw["u_ref"]
    Cf = np.zeros((B, 17, 17), np.float32) if kw["C_f"] is None else kw["C_f"]
    cf = np.zeros((B, 17), np.float32) if kw["c_f"] is None else kw["c_f"]
    c0 = O.objective(X0, d["U_init"], zx, zu, d["C"], d["c"], Cf, cf)
    assert np.all(r["best_cost"] <= c0 + 1e-6 * np.abs(c0))
    assert np.all(r["iters"] >= 1)


def test_rotor13_ragged_batch_and_many_step_sizes():
    """B = 13 (a CTA with unused element slots), eight step sizes (eight
    candidate lanes and nine trajectory slots), replayed against the oracle."""
    d = load("r13_cfg2_b32_t10")
    alphas = (1.0, 0.8, 0.6, 0.5, 0.3, 0.2, 0.1, 0.05)
    r = _gpu_solve(d, B=13, alphas=alphas, max_iter=4)
    o64, reals = _realisations(d, r["trace"], B=13, alphas=alphas, max_iter=4)
    for key in ("X", "U"):
        assert not _check_rounding(r[key], o64, reals, key, TOL_XU), key
    assert (r["trace"][:, 0] >= 0).any()


def test_rotor13_single_step_horizon():
    d = load("r13_cfg1_b16_t5")
    dd = dict(d)
    dd["U_init"] = d["U_init"][:, :1]
    dd["C"] = d["C"][:, :1]
    dd["c"] = d["c"][:, :1]
    r = _gpu_solve(dd, max_iter=3)
    o32, _ = _oracle(dd, r["trace"], max_iter=3)
    assert max_rel(r["X"], o32["X"]) <= TOL_XU
    assert max_rel(r["U"], o32["U"]) <= TOL_XU


def test_rotor13_fastmpc_autograd_surface():
    """FastMPC(13, 4, T) forward equals the entry point's solve, and autograd
    returns the backward entry point's gradients of x0, C, c."""
    d = load("r13_cfg1_b16_t5")
    B, T = d["U_init"].shape[:2]
    kw = case_kwargs(d)
    lo = torch.zeros(T, B, 4, device=DEV)
    hi = torch.ones(T, B, 4, device=DEV)
    m = mpc_compat.FastMPC(13, 4, T, u_lower=lo, u_upper=hi, lqr_iter=kw["max_iter"], eps=kw["reg"])
    x0 = _t(d["x0"]).requires_grad_(True)
    C = _t(d["C"]).permute(1, 0, 2, 3).contiguous().requires_grad_(True)
    c = _t(d["c"]).permute(1, 0, 2).contiguous().requires_grad_(True)
    X, U, _ = m(x0, mpc_compat.QuadCost(C, c), type("Dx", (), {"dt": kw["dt"]})())
    ref = _gpu_solve(d)
    assert np.array_equal(X.detach().permute(1, 0, 2).cpu().numpy(), ref["X"])
    assert np.array_equal(U.detach().permute(1, 0, 2).cpu().numpy(), ref["U"])
    gX = _t(d["gX"]).permute(1, 0, 2)
    gU = _t(d["gU"]).permute(1, 0, 2)
    ((X * gX).sum() + (U * gU).sum()).backward()
    g = _gpu_backward(d, ref["X"], ref["U"], ref["tight"], kw)
    assert np.array_equal(x0.grad.cpu().numpy(), g["grad_x0"])
    assert np.array_equal(C.grad.permute(1, 0, 2, 3).cpu().numpy(), g["grad_C"])
    assert np.array_equal(c.grad.permute(1, 0, 2).cpu().numpy(), g["grad_c"])


def test_rotor13_rollout_config_prefix():
    """512 elements of the training-scale configuration (T = 20, 5
    iterations, box [0, 1]): the kernel's decisions replayed in the oracle."""
    cfg, inp = wl.rotor13_config_inputs("rollout_b16384_t20", B=512)
    d = dict(inp, dt=np.array(wl.DT), max_iter=np.array(cfg["max_iter"]),
             alphas=np.array(cfg["alphas"], np.float32), bounds=np.array(True), reg=np.array(1e-6),
             u_min=wl.U_MIN13, u_max=wl.U_MAX13)
    r = _gpu_solve(d)
    assert np.isfinite(r["X"]).all() and np.isfinite(r["U"]).all()
    o64, reals = _realisations(d, r["trace"])
    for key in ("X", "U"):
        fails = _check_rounding(r[key], o64, reals, key, TOL_XU)
        assert not fails, (key, fails[:5])
    well = rel_per_elem(reals[0]["X"], o64["X"]) <= WELL_CONDITIONED
    assert well.mean() > 0.5


def test_rotor13_nonfinite_elements_are_isolated():
    """As the 10-state test: a NaN x0 and an infinite cost weight stay
    confined to their elements (rejected first step, U_init kept), and the
    rest of the batch is bit-identical to the run without them."""
    d = load("r13_cfg1_b16_t5")
    bad = dict(d)
    bad["x0"] = d["x0"].copy()
    bad["x0"][3, 0] = np.nan
    bad["C"] = d["C"].copy()
    bad["C"][7, 2, 1, 1] = np.inf
    r = _gpu_solve(bad)
    r0 = _gpu_solve(d)
    others = [b for b in range(16) if b not in (3, 7)]
    for k in ("X", "U", "tight", "trace"):
        assert np.array_equal(r[k][others], r0[k][others]), k
    for b in (3, 7):
        assert r["trace"][b, 0] < 0 and (r["trace"][b, 1:] == -128).all()
        assert np.array_equal(r["U"][b], d["U_init"][b])
    assert r["status"][3] & 2 and np.isnan(r["best_cost"][3])
    assert np.isinf(r["best_cost"][7])


def test_rotor13_register_tiers_are_bit_identical():
    """The solve runs a 2-CTA-per-SM register budget for grids of one wave
    and a 3-CTA one beyond (B > 2368); both give the same bits: the first
    512 elements of a B=2400 solve equal a B=512 solve (the generator's
    batches share prefixes), the backward likewise."""
    cfg, inp = wl.rotor13_config_inputs("rollout_b16384_t20", B=2400)
    t = lambda a: _t(a)
    lo, hi = _t(wl.U_MIN13), _t(wl.U_MAX13)
    gX, gU = wl.make_backward_seeds(2400, cfg["T"], nx=wl.NX13)
    outs = []
    for B in (2400, 512):
        o = nat.rotor13_solve(t(inp["x0"][:B]), t(inp["U_init"][:B]), t(inp["C"][:B]), t(inp["c"][:B]),
                              u_min=lo, u_max=hi, dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"],
                              want_trace=True)
        g = nat.rotor13_backward(o["X"], o["U"], t(inp["C"][:B]), t(gX[:B]), t(gU[:B]), tight=o["tight"],
                                 dt=wl.DT)
        outs.append(({k: v[:512].cpu().numpy() for k, v in o.items()},
                     {k: v[:512].cpu().numpy() for k, v in g.items()}))
    (o1, g1), (o2, g2) = outs
    for k in o2:
        assert np.array_equal(o1[k], o2[k], equal_nan=True), k
    for k in g2:
        assert np.array_equal(g1[k], g2[k], equal_nan=True), k
