"""Pins of the FastMPC-numerics oracle (oracle/fastmpc_oracle.py).

The reference FastMPC extension cannot be built as a whole here (it needs
libtorch); its CUDA kernels are checked against the B200 kernels on the GPU
(tests/test_gpu_fastmpc_reference.py). On the CPU the restatement is pinned
piece by piece against mathematics the reference code implements:
- the model: the Jacobian is I + dt times the exact derivative of the
  continuous dynamics (central differences in fp64), and the two step forms
  (rotation matrix and cross product) agree and keep the quaternion unit;
- the Riccati pass and line search: on a linear-quadratic problem one
  iteration with alpha = 1 lands on the closed-form optimum (a dense KKT solve
  in fp64), and with a separable control box it lands on the box optimum;
- the adjoint: on the same problem the gradients equal central differences of
  the solution's loss (directional, symmetric cost perturbations);
- pnqp4 itself is pinned to mpc.pytorch's pnqp by test_oracle_golden.py.
"""

import numpy as np
import pytest

import oracle as O

F32 = np.float32


def _xdot64(x, u, mass=0.752, g=-9.8066):
    """Continuous CTBR dynamics in fp64 with the polynomial rotation of q."""
    qw, qx, qy, qz = x[3:7]
    vx, vy, vz = x[7:10]
    fc, wx, wy, wz = u
    dq = 0.5 * np.array([-qx * wx - qy * wy - qz * wz,
                         qw * wx + qy * wz - qz * wy,
                         qw * wy - qx * wz + qz * wx,
                         qw * wz + qx * wy - qy * wx])
    r13 = 2 * (qx * qz + qw * qy)
    r23 = 2 * (qy * qz - qw * qx)
    r33 = qw * qw - qx * qx - qy * qy + qz * qz
    dv = np.array([r13, r23, r33]) * fc / mass + np.array([0, 0, g])
    return np.concatenate([[vx, vy, vz], dq, dv])


def test_jacobian_is_euler_jacobian_of_continuous_dynamics():
    rng = np.random.default_rng(0)
    dt = 0.05
    for _ in range(20):
        x = rng.normal(size=10)
        u = np.array([rng.uniform(0, 30), *rng.normal(size=3)])
        A, B = O.fm_jacobian(x[None].astype(F32), u[None].astype(F32), dt)
        h = 1e-6
        Jx = np.stack([(_xdot64(x + h * e, u) - _xdot64(x - h * e, u)) / (2 * h) for e in np.eye(10)], axis=1)
        Ju = np.stack([(_xdot64(x, u + h * e) - _xdot64(x, u - h * e)) / (2 * h) for e in np.eye(4)], axis=1)
        np.testing.assert_allclose(A[0], np.eye(10) + dt * Jx, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(B[0], dt * Ju, rtol=1e-5, atol=1e-5)


def test_step_forms_agree_and_renormalise():
    rng = np.random.default_rng(1)
    x = np.zeros((64, 10), F32)
    x[:, :3] = rng.normal(size=(64, 3))
    q = rng.normal(size=(64, 4))
    x[:, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True)
    x[:, 7:] = rng.normal(size=(64, 3))
    u = np.concatenate([rng.uniform(0, 30, (64, 1)), rng.normal(size=(64, 3))], axis=1).astype(F32)
    a = O.fm_step(x, u, 0.05)
    b = O.fm_rollout_step(x, u, 0.05)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(np.linalg.norm(a[:, 3:7], axis=1), 1.0, atol=1e-6)
    # the unnormalised product: |q (x) exp_map| = |q| for unit exp_map
    assert np.abs(np.linalg.norm(a[:, 3:7], axis=1) - 1).max() < 1e-6


# ---- a linear-quadratic problem -----------------------------------------------

NXL, NUL = 6, 4


def _lq_problem(B, T, seed, sep=False):
    rng = np.random.default_rng(seed)
    A = np.eye(NXL) + 0.1 * rng.normal(size=(B, T, NXL, NXL))
    if sep:
        # orthogonal control columns and a scaled-identity terminal cost keep
        # B^T V B diagonal at T = 1, so the control box QP separates
        Bm = np.zeros((B, T, NXL, NUL))
        for i in range(NUL):
            Bm[:, :, i, i] = rng.uniform(0.5, 1.5, (B, T))
    else:
        Bm = 0.3 * rng.normal(size=(B, T, NXL, NUL))
    n = NXL + NUL
    G = rng.normal(size=(B, T, n, n)) * 0.3
    C = G @ np.swapaxes(G, -1, -2) / n + np.eye(n) * rng.uniform(0.5, 2.0, (B, T, n))[..., None]
    if sep:
        C[:, :, :NXL, NXL:] = 0
        C[:, :, NXL:, :NXL] = 0
        C[:, :, NXL:, NXL:] = np.eye(NUL) * rng.uniform(0.5, 2.0, (B, T, NUL))[..., None]
    c = rng.normal(size=(B, T, n))
    Cf = np.zeros((B, n, n))
    Cf[:, :NXL, :NXL] = np.eye(NXL) * 2.0
    x0 = rng.normal(size=(B, NXL))
    f = lambda a: np.asarray(a, F32)
    return f(A), f(Bm), f(C), f(c), f(Cf), f(x0)


def _linear_model(A, Bm):
    state = {"t": 0}

    def step(x, u, dt):
        # the rollouts call step once per t in order; t is recovered from a counter
        t = state["t"] % A.shape[1]
        state["t"] += 1
        s = np.zeros_like(x)
        for j in range(NXL):
            s = s + A[:, t, :, j] * x[:, j, None]
        for j in range(NUL):
            s = s + Bm[:, t, :, j] * u[:, j, None]
        return s.astype(F32)

    def jac(X, U, dt):
        return A, Bm

    return step, jac


def _kkt_optimum(A, Bm, C, c, Cf, x0):
    """Minimiser of sum_t 1/2 z^T C z + c^T z + 1/2 x_T^T Cf_xx x_T over U
    (fp64, dense): X = S x0 + M U."""
    B, T = A.shape[:2]
    out = np.empty((B, T, NUL))
    for b in range(B):
        S = [np.eye(NXL)]
        M = [np.zeros((NXL, T * NUL))]
        for t in range(T):
            S.append(A[b, t] @ S[-1])
            m = A[b, t] @ M[-1]
            m[:, t * NUL:(t + 1) * NUL] += Bm[b, t]
            M.append(m)
        H = np.zeros((T * NUL, T * NUL))
        g = np.zeros(T * NUL)
        for t in range(T + 1):
            Ct = Cf[b].astype(np.float64) if t == T else C[b, t].astype(np.float64)
            ct = np.zeros(NXL + NUL) if t == T else c[b, t].astype(np.float64)
            E = np.zeros((NXL + NUL, T * NUL))
            E[:NXL] = M[t]
            if t < T:
                E[NXL:, t * NUL:(t + 1) * NUL] = np.eye(NUL)
            z0 = np.concatenate([S[t] @ x0[b], np.zeros(NUL)])
            Cs = 0.5 * (Ct + Ct.T)
            H += E.T @ Cs @ E
            g += E.T @ (Cs @ z0 + ct)
        out[b] = np.linalg.solve(H, -g).reshape(T, NUL)
    return out


def test_one_iteration_reaches_lq_optimum():
    B, T = 6, 5
    A, Bm, C, c, Cf, x0 = _lq_problem(B, T, 3)
    step, jac = _linear_model(A, Bm)
    r = O.fm_solve(x0, np.zeros((B, T, NUL), F32), C, c, C_f=Cf, dt=0.05, max_iter=1, reg=1e-9,
                   step=step, rollout_step=step, jacobian=jac)
    assert (r["trace"][:, 0] == 0).all()
    np.testing.assert_allclose(r["U"], _kkt_optimum(A, Bm, C, c, Cf, x0), rtol=1e-3, atol=1e-4)


def test_separable_box_lands_on_box_optimum():
    B, T = 32, 1
    A, Bm, C, c, Cf, x0 = _lq_problem(B, T, 4, sep=True)
    step, jac = _linear_model(A, Bm)
    lo = np.full(NUL, -0.3, F32)
    hi = np.full(NUL, 0.3, F32)
    r = O.fm_solve(x0, np.zeros((B, T, NUL), F32), C, c, C_f=Cf, u_min=lo, u_max=hi, dt=0.05, max_iter=1,
                   reg=1e-9, step=step, rollout_step=step, jacobian=jac)
    free = _kkt_optimum(A, Bm, C, c, Cf, x0)
    want = np.clip(free, -0.3, 0.3)
    np.testing.assert_allclose(r["U"], want, rtol=1e-4, atol=1e-5)
    assert (r["tight"] == (np.abs(free) > 0.3)).all()
    assert r["tight"].any() and (~r["tight"]).any()


def _loss(x0, C, c, Cf, A, Bm, gX, gU):
    step, jac = _linear_model(A, Bm)
    B, T = C.shape[:2]
    r = O.fm_solve(x0, np.zeros((B, T, NUL), F32), C, c, C_f=Cf, dt=0.05, max_iter=1, reg=1e-9,
                   step=step, rollout_step=step, jacobian=jac)
    assert (r["trace"][:, 0] == 0).all()
    return float(np.sum(r["X"].astype(np.float64) * gX) + np.sum(r["U"].astype(np.float64) * gU)), r


def test_adjoint_matches_central_differences():
    B, T = 4, 4
    A, Bm, C, c, Cf, x0 = _lq_problem(B, T, 5)
    rng = np.random.default_rng(6)
    gX = rng.normal(size=(B, T + 1, NXL)).astype(F32)
    gU = rng.normal(size=(B, T, NUL)).astype(F32)
    _, r = _loss(x0, C, c, Cf, A, Bm, gX, gU)
    _, jac = _linear_model(A, Bm)
    g = O.fm_backward(r["X"], r["U"], r["X_lin"], r["U_lin"], C, gX, gU, r["tight"], C_f=Cf, reg=1e-9,
                      jacobian=jac)
    # x0 and c: the solution is linear in them, a large step is exact
    for name, base, grad, eps in (("x0", x0, g["x0"], 0.5), ("c", c, g["c"], 0.5)):
        d = rng.normal(size=base.shape).astype(F32)
        args = dict(x0=x0, C=C, c=c)
        lp = _loss(**{**args, name: (base + eps * d).astype(F32)}, Cf=Cf, A=A, Bm=Bm, gX=gX, gU=gU)[0]
        lm = _loss(**{**args, name: (base - eps * d).astype(F32)}, Cf=Cf, A=A, Bm=Bm, gX=gX, gU=gU)[0]
        fd = (lp - lm) / (2 * eps)
        an = float(np.sum(grad.astype(np.float64) * d))
        assert abs(fd - an) <= 2e-3 * max(1.0, abs(an)), (name, fd, an)
    # C: symmetric directions, central differences
    d = rng.normal(size=C.shape)
    d = (0.5 * (d + np.swapaxes(d, -1, -2))).astype(F32)
    eps = 1e-2
    lp = _loss(x0, (C + eps * d).astype(F32), c, Cf, A, Bm, gX, gU)[0]
    lm = _loss(x0, (C - eps * d).astype(F32), c, Cf, A, Bm, gX, gU)[0]
    fd = (lp - lm) / (2 * eps)
    an = float(np.sum(g["C"].astype(np.float64) * d))
    assert abs(fd - an) <= 1e-2 * max(1.0, abs(an)), (fd, an)


def test_batch_convergence_flag_and_replay():
    import ilqr_workload as wl
    d = wl.make_inputs(6, 5, seed=2)
    lo = np.array([0, -10, -10, -4], F32)
    hi = np.array([34, 10, 10, 4], F32)
    r = O.fm_solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=lo, u_max=hi, max_iter=9)
    # a replay of its own decisions and stop reproduces the run bit for bit
    rr = O.fm_solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=lo, u_max=hi, max_iter=9, forced=r["trace"],
                    forced_stop=r["iters_run"])
    for k in ("X", "U", "tight", "X_lin", "U_lin"):
        assert np.array_equal(rr[k], r[k]), k
    # a forced stop after the first check (iteration 4) ends the run there
    rs = O.fm_solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=lo, u_max=hi, max_iter=9, forced=r["trace"],
                    forced_stop=4)
    assert rs["iters_run"] == 4 and rs["converged"]
    assert (rs["trace"][:, 4:] == O.NOT_RUN).all()


@pytest.mark.parametrize("tight_none", [False, True])
def test_adjoint_mask_zeroes_clamped_directions(tight_none):
    """With a tight entry the adjoint's dU is zero there (its row of K and its
    k are zero): the clamped control does not move."""
    B, T = 5, 4
    A, Bm, C, c, Cf, x0 = _lq_problem(B, T, 8)
    rng = np.random.default_rng(9)
    tight = rng.uniform(size=(B, T, NUL)) < 0.4
    gX = rng.normal(size=(B, T + 1, NXL)).astype(F32)
    gU = rng.normal(size=(B, T, NUL)).astype(F32)
    _, jac = _linear_model(A, Bm)
    X = rng.normal(size=(B, T + 1, NXL)).astype(F32)
    U = rng.normal(size=(B, T, NUL)).astype(F32)
    g = O.fm_backward(X, U, X, U, C, gX, gU, None if tight_none else tight, C_f=Cf, jacobian=jac)
    if tight_none:
        assert np.abs(g["u_ref"]).min() > 0
    else:
        assert (g["u_ref"][tight] == 0).all() and (g["K"][tight] == 0).all() and (g["k"][tight] == 0).all()
