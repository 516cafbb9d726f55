"""Known-answer checks of the oracle against calculus (CPU, float64):
Jacobians against central differences, and the implicit-differentiation
gradients against finite differences of the converged solve. The GPU kernels
are checked against the oracle elsewhere (Jacobians bit for bit)."""

import numpy as np
import pytest

import oracle as O
from oracle.diffmpc_oracle import quat_mult, rotate_quat


def _central_jacobian(f, x, u, eps=1e-6):
    nb, nx = x.shape
    nu = u.shape[1]
    Jx = np.zeros((nb, f(x, u).shape[1], nx))
    Ju = np.zeros((nb, f(x, u).shape[1], nu))
    for j in range(nx):
        e = np.zeros(nx)
        e[j] = eps
        Jx[:, :, j] = (f(x + e, u) - f(x - e, u)) / (2 * eps)
    for j in range(nu):
        e = np.zeros(nu)
        e[j] = eps
        Ju[:, :, j] = (f(x, u + e) - f(x, u - e)) / (2 * eps)
    return Jx, Ju


def _ctbr_xdot(x, u):
    """Continuous CTBR dynamics (drone.py:409-465 before discretisation):
    p' = v, q' = 1/2 q (x) (0, w), v' = R(q) (0, 0, fc) / m + g."""
    q = x[:, 3:7].T
    w = np.concatenate([np.zeros((1, x.shape[0])), u[:, 1:4].T])
    qd = 0.5 * quat_mult(q, w)
    thrust = np.concatenate([np.zeros((2, x.shape[0])), u[:, 0][None, :]])
    vd = rotate_quat(q, thrust) / O.MASS + np.array([0.0, 0.0, O.GRAV_Z])[:, None]
    return np.concatenate([x[:, 7:10].T, qd, vd]).T


def test_ctbr_jacobian_is_the_euler_jacobian_of_the_continuous_dynamics():
    """The reference linearises the continuous dynamics (A = I + dt df/dx,
    B = dt df/du), not its exponential-map step; central differences of the
    continuous dynamics confirm the restated Jacobian, with one exception the
    restatement keeps for parity: the reference's aux_q_dot_dw_3
    (acmpc_public-master/diff_mpc_drones/drone.py:229-232) has -1 in row 1,
    column 2, so its dq_x/dw_z is -qy/2 where the derivative of
    1/2 q (x) (0, w) is +qy/2."""
    rng = np.random.default_rng(0)
    x = rng.normal(size=(32, 10))
    x[:, 3:7] /= np.linalg.norm(x[:, 3:7], axis=1, keepdims=True)
    u = np.concatenate([rng.uniform(0, 34, (32, 1)), rng.uniform(-10, 10, (32, 3))], axis=1)
    dt = 0.05
    A, Bm = O.drone_jacobian(x, u, dt)
    Jx, Ju = _central_jacobian(_ctbr_xdot, x, u)
    assert np.abs((A - np.eye(10)) / dt - Jx).max() <= 1e-6 * max(1.0, np.abs(Jx).max())
    Jb = Bm / dt
    tol = 1e-6 * max(1.0, np.abs(Ju).max())
    assert np.allclose(Jb[:, 4, 3], -0.5 * x[:, 5]) and np.allclose(Ju[:, 4, 3], 0.5 * x[:, 5])
    Jb[:, 4, 3] = -Jb[:, 4, 3]
    assert np.abs(Jb - Ju).max() <= tol


def test_rotor13_jacobian_is_the_exact_step_jacobian():
    rng = np.random.default_rng(1)
    x = rng.normal(size=(32, 13))
    x[:, 3:7] /= np.linalg.norm(x[:, 3:7], axis=1, keepdims=True)
    u = rng.uniform(0, 1, (32, 4))
    dt = 0.05
    A, Bm = O.rotor13_jacobian(x, u, dt)
    Jx, Ju = _central_jacobian(lambda a, b: O.rotor13_step(a, b, dt), x, u)
    assert np.abs(A - Jx).max() <= 1e-6 * max(1.0, np.abs(Jx).max())
    assert np.abs(Bm - Ju).max() <= 1e-6 * max(1.0, np.abs(Ju).max())


def _linear_model(nx, nu, seed):
    rng = np.random.default_rng(seed)
    A = np.eye(nx) + 0.1 * rng.normal(size=(nx, nx))
    B = 0.2 * rng.normal(size=(nx, nu))
    step = lambda x, u, dt: x @ A.T.astype(x.dtype) + u @ B.T.astype(x.dtype)

    def jac(x, u, dt):
        n = x.shape[0]
        return (np.broadcast_to(A.astype(x.dtype), (n, nx, nx)).copy(),
                np.broadcast_to(B.astype(x.dtype), (n, nx, nu)).copy())

    return O.Model("linear", nx, nu, step, jac)


@pytest.mark.parametrize("seed", [0, 1])
def test_implicit_diff_matches_finite_differences(seed):
    """Unconstrained problem with linear dynamics: the iLQR fixed point is the
    exact optimum, so the implicit-diff gradients of L = <gX, X*> + <gU, U*>
    (ILQRSolve.backward semantics) equal central differences of the
    converged solve with respect to x0, c and C (symmetric perturbations)."""
    nx, nu, T, nb = 4, 2, 6, 3
    n = nx + nu
    model = _linear_model(nx, nu, seed)
    rng = np.random.default_rng(10 + seed)
    G = rng.normal(size=(nb, T, n, n))
    C = G @ np.swapaxes(G, -1, -2) / n + np.eye(n)
    c = rng.normal(size=(nb, T, n))
    x0 = rng.normal(size=(nb, nx))
    U0 = np.zeros((nb, T, nu))
    gX = rng.normal(size=(nb, T + 1, nx))
    gU = rng.normal(size=(nb, T, nu))
    kw = dict(dt=0.05, max_iter=30, reg=1e-9, dtype=np.float64, model=model, alphas=(1.0, 0.5, 0.25))
    forced = None  # the perturbed solves replay the base solve's decisions

    def loss(x0_, C_, c_):
        r = O.solve(x0_, U0, C_, c_, forced=forced, **kw)
        return np.sum(gX * r["X"]) + np.sum(gU * r["U"]), r

    _, r = loss(x0, C, c)
    forced = r["trace"]
    g = O.backward(r["X"], r["U"], C, None, None, None, r["tight"], gX, gU, 0.05, 1e-9,
                   dtype=np.float64, model=model)
    eps = 1e-5
    checks = []
    for (b, i) in [(0, 0), (1, 2), (2, 3)]:
        xp, xm = x0.copy(), x0.copy()
        xp[b, i] += eps
        xm[b, i] -= eps
        checks.append(((loss(xp, C, c)[0] - loss(xm, C, c)[0]) / (2 * eps), g["grad_x0"][b, i]))
    for (b, t, i) in [(0, 0, 1), (1, 3, 4), (2, 5, 0)]:
        cp, cm = c.copy(), c.copy()
        cp[b, t, i] += eps
        cm[b, t, i] -= eps
        checks.append(((loss(x0, C, cp)[0] - loss(x0, C, cm)[0]) / (2 * eps), g["grad_c"][b, t, i]))
    for (b, t, i, j) in [(0, 1, 0, 0), (1, 2, 1, 4), (2, 4, 3, 5)]:
        Cp, Cm = C.copy(), C.copy()
        for (a, d) in {(i, j), (j, i)}:
            Cp[b, t, a, d] += eps
            Cm[b, t, a, d] -= eps
        fd = (loss(x0, Cp, c)[0] - loss(x0, Cm, c)[0]) / (2 * eps)
        an = g["grad_C"][b, t, i, j] + (g["grad_C"][b, t, j, i] if i != j else 0.0)
        checks.append((fd, an))
    for fd, an in checks:
        assert abs(fd - an) <= 1e-5 * max(1.0, abs(fd)), (fd, an)
