"""TEST INFRASTRUCTURE ONLY -- numpy restatement of DiffMPC + DroneDx (CTBR model).

Every function cites the reference lines it restates (paths relative to the
reference project root). The arithmetic follows the reference's operation
order where it is observable (elementwise expressions are evaluated in the same
order, so they round identically in float32); reductions inside matmul /
einsum / LAPACK have implementation-defined order in the reference and differ
here only at the rounding level.

Decision traces. The reference's line search makes two discrete decisions per
element and iteration: the argmin over step sizes (first minimum, NaN first,
controller.py:382) and the strict-improvement test (controller.py:396). After
the first Newton step the candidate costs are frequently equal to within fp32
rounding, so those decisions are rounding noise in *any* fp32 implementation
(including the reference against itself in fp64). `solve` therefore records a
trace and can replay one:

    trace[b, i] = j          element b accepted candidate j at iteration i
    trace[b, i] = -(j + 1)   element b rejected (argmin j): X, U, cost kept
    trace[b, i] = -128       iteration i was not run for element b

Replaying a trace (``forced=``) makes the oracle take exactly those
decisions (a rejection keeps X, U and continues; -128 stops), so the
remaining arithmetic can be compared at a strict tolerance.

Per-element freezing. When an element fails to improve, its X, U and best
cost are unchanged, so a deterministic implementation recomputes identical
candidates on every later iteration and never improves it again; the global
loop exit (controller.py:402-406) then changes no element's X/U. Free-running,
the oracle freezes each element at its first rejection and reconstructs the
reference's global ``converged`` flag from the per-element stall iteration
and gap. (The reference's own CPU reductions are not bit-stable across
iterations, so on rounding-level ties it can occasionally re-improve a
rejected element; a recorded trace reproduces that under replay.)
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
NX, NU, N = 10, 4, 14
MASS = 0.752          # drone.py:166
GRAV_Z = -9.8066      # drone.py:187
NOT_RUN = -128

DEFAULT_ALPHAS = (1.0, 0.8, 0.5, 0.2, 0.1)   # controller.py:211


def _f(x, dtype):
    return np.asarray(x, dtype=dtype)


# --------------------------------------------------------------------------
# Quadrotor CTBR model (acmpc_public-master/diff_mpc_drones/drone.py)
# --------------------------------------------------------------------------

def quat_mult(q1, q2):
    """drone.py:28-33. q1, q2: [4, B] (component-major, as the reference)."""
    return np.stack([
        q2[0] * q1[0] - q2[1] * q1[1] - q2[2] * q1[2] - q2[3] * q1[3],
        q2[0] * q1[1] + q2[1] * q1[0] - q2[2] * q1[3] + q2[3] * q1[2],
        q2[0] * q1[2] + q2[2] * q1[0] + q2[1] * q1[3] - q2[3] * q1[1],
        q2[0] * q1[3] - q2[1] * q1[2] + q2[2] * q1[1] + q2[3] * q1[0]])


def exp_map(w, dt):
    """drone.py:18-26. w: [3, B]. torch.nn.functional.normalize divides by
    max(norm, 1e-12)."""
    dtype = w.dtype
    w_norm = np.sqrt(np.sum(w * w, axis=0, dtype=dtype)).astype(dtype)
    w_normalized = w / np.maximum(w_norm, dtype.type(1e-12))
    half = w_norm * dtype.type(dt * 0.5)
    s = np.sin(half)
    return np.stack([np.cos(half), w_normalized[0] * s, w_normalized[1] * s,
                     w_normalized[2] * s])


def rotate_quat(q1, v1):
    """drone.py:145-156: imaginary part of q1 (x) [0, v1] (x) conj(q1)."""
    zero = np.zeros((1, q1.shape[1]), dtype=q1.dtype)
    conj = np.stack([q1[0], -q1[1], -q1[2], -q1[3]])
    ans = quat_mult(quat_mult(q1, np.concatenate([zero, v1])), conj)
    return np.stack([ans[1], ans[2], ans[3]])


def drone_step(x, u, dt, mass=MASS):
    """DroneDx.forward_CTBR (drone.py:409-465). x [B,10], u [B,4] -> [B,10].

    p+ = p + dt v;  q+ = q (x) exp(w, dt) (no renormalisation);
    v+ = v + dt (R(q)[0,0,fc]/m + g).
    """
    dtype = x.dtype
    dtt = dtype.type(dt)
    p = x[:, 0:3].T
    q = x[:, 3:7].T
    v = x[:, 7:10].T
    w = u[:, 1:4].T
    fc = u[:, 0]
    new_p = p + dtt * v
    new_q = quat_mult(q, exp_map(w, dt))
    n_b = x.shape[0]
    thrust = np.concatenate([np.zeros((2, n_b), dtype=dtype), fc[None, :]])
    g = np.array([0.0, 0.0, GRAV_Z], dtype=dtype)[:, None]
    new_v = v + dtt * (rotate_quat(q, thrust) / dtype.type(mass) + g)
    return np.concatenate([new_p, new_q, new_v]).T.copy()


def drone_jacobian(x, u, dt, mass=MASS):
    """DroneDx.grad_input / get_A_B_mat_CTBR (drone.py:489-540).

    Euler Jacobian of the continuous CTBR dynamics (not of the exp-map step):
    A = I + dt * J_x, B = dt * J_u. x [B,10], u [B,4] -> A [B,10,10], B [B,10,4].
    """
    dtype = x.dtype
    dtt = dtype.type(dt)
    m = dtype.type(mass)
    nb = x.shape[0]
    R = np.zeros((nb, NX, NX), dtype=dtype)
    S = np.zeros((nb, NX, NU), dtype=dtype)
    half = dtype.type(0.5)
    two = dtype.type(2.0)
    # d p_dot / d v = I3 (drone.py:504)
    for i in range(3):
        R[:, i, 7 + i] = 1.0
    # d q_dot / d q = 0.5 * Omega(w) (drone.py:308-314, aux_d_q_dot_dq_* at :236-254)
    wx, wy, wz = u[:, 1], u[:, 2], u[:, 3]
    zq = np.zeros_like(wx)
    cols = [np.stack([zq, wx, wy, wz]), np.stack([-wx, zq, -wz, wy]),
            np.stack([-wy, wz, zq, -wx]), np.stack([-wz, -wy, wx, zq])]
    for j in range(4):
        R[:, 3:7, 3 + j] = (half * cols[j]).T
    # d v_dot / d q = 2 * aux_k @ (q * fc / m) (drone.py:316-326, aux at :257-271)
    q = x[:, 3:7]
    fc = u[:, 0]
    qf = (q * fc[:, None]) / m
    q0, q1, q2, q3 = qf[:, 0], qf[:, 1], qf[:, 2], qf[:, 3]
    vcols = [np.stack([q2, -q1, q0]), np.stack([q3, -q0, -q1]),
             np.stack([q0, q3, -q2]), np.stack([q1, q2, q3])]
    for j in range(4):
        R[:, 7:10, 3 + j] = (two * vcols[j]).T
    # d v_dot / d fc = (q^T aux_dv_k q) / m (drone.py:336-344, aux at :288-301)
    a0, a1, a2, a3 = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    d1 = (a2 * a0 + a3 * a1 + a0 * a2 + a1 * a3)
    d2 = (-a1 * a0 + -a0 * a1 + a3 * a2 + a2 * a3)
    d3 = (a0 * a0 + -a1 * a1 + -a2 * a2 + a3 * a3)
    S[:, 7, 0] = d1 / m
    S[:, 8, 0] = d2 / m
    S[:, 9, 0] = d3 / m
    # d q_dot / d w = 0.5 * aux_q_dot_dw_k @ q (drone.py:305-306, aux at :220-233)
    wcols = [np.stack([-a1, a0, a3, -a2]), np.stack([-a2, -a3, a0, a1]),
             np.stack([-a3, -a2, -a1, a0])]
    for j in range(3):
        S[:, 3:7, 1 + j] = (half * wcols[j]).T
    A = R * dtt + np.eye(NX, dtype=dtype)[None]
    Bm = S * dtt
    return A, Bm


class Model:
    """A discrete dynamics model as the solver sees it (DiffMPC's f_dyn and
    f_dyn_jac, controller.py:147-160): step(x [B,nx], u [B,nu], dt) -> x_next
    and jacobian(x, u, dt) -> (A [B,nx,nx], B [B,nx,nu])."""

    def __init__(self, name, nx, nu, step, jacobian):
        self.name, self.nx, self.nu = name, nx, nu
        self.step, self.jacobian = step, jacobian

    def __repr__(self):
        return f"Model({self.name}, nx={self.nx}, nu={self.nu})"


DRONE10 = Model("drone_ctbr10", NX, NU, drone_step, drone_jacobian)


def rollout(x0, U, dt, model=None):
    """controller.py:578-603 (open-loop rollout)."""
    model = model or DRONE10
    nb, T, _ = U.shape
    X = np.empty((nb, T + 1, model.nx), dtype=x0.dtype)
    X[:, 0] = x0
    xt = x0
    for t in range(T):
        xt = model.step(xt, U[:, t], dt)
        X[:, t + 1] = xt
    return X


def linearize(X, U, dt, model=None):
    """controller.py:607-622: the model's Jacobian at every (X_t, U_t)."""
    model = model or DRONE10
    nx, nu = model.nx, model.nu
    nb, T = U.shape[:2]
    A, Bm = model.jacobian(X[:, :-1].reshape(-1, nx), U.reshape(-1, nu), dt)
    return A.reshape(nb, T, nx, nx), Bm.reshape(nb, T, nx, nu)


# --------------------------------------------------------------------------
# Quadratic cost (DifferentialMPC/cost.py)
# --------------------------------------------------------------------------

def objective(X, U, x_ref, u_ref, C, c, C_f, c_f):
    """GeneralQuadCost.objective_pure (cost.py:173-233). All inputs batched."""
    dtype = X.dtype
    T = U.shape[1]
    tau = np.concatenate([X[:, :T] - x_ref[:, :T], U - u_ref], axis=-1)
    half = dtype.type(0.5)
    run_q = np.einsum("bti,btij,btj->b", tau, C, tau).astype(dtype)
    run_l = np.einsum("bti,bti->b", c, tau).astype(dtype)
    tauN = np.concatenate([X[:, -1] - x_ref[:, -1],
                           np.zeros((X.shape[0], U.shape[-1]), dtype=dtype)], axis=-1)
    fin_q = np.einsum("bi,bij,bj->b", tauN, C_f, tauN).astype(dtype)
    fin_l = np.einsum("bi,bi->b", c_f, tauN).astype(dtype)
    return (half * run_q + run_l) + (half * fin_q + fin_l)


def quadraticize(X, U, x_ref, u_ref, C, c, C_f, c_f):
    """GeneralQuadCost.quadraticize (cost.py:130-171)."""
    dtype = X.dtype
    T = U.shape[1]
    tau = np.concatenate([X[:, :T] - x_ref[:, :T], U - u_ref], axis=-1)
    l_tau = np.einsum("btij,btj->bti", C, tau).astype(dtype) + c
    nx = X.shape[-1]
    tauN = np.concatenate([X[:, -1] - x_ref[:, -1],
                           np.zeros((X.shape[0], U.shape[-1]), dtype=dtype)], axis=-1)
    lN = np.einsum("bij,bj->bi", C_f, tauN).astype(dtype) + c_f
    return (l_tau[..., :nx], l_tau[..., nx:], C[..., :nx, :nx],
            C[..., :nx, nx:], C[..., nx:, nx:], lN[..., :nx], C_f[..., :nx, :nx])


# --------------------------------------------------------------------------
# Linear algebra helpers (4x4 Cholesky, as LAPACK's unblocked potf2 / potrs)
# --------------------------------------------------------------------------

def chol4(M):
    """Lower Cholesky factor of [B,n,n] reading the lower triangle only
    (torch.linalg.cholesky semantics). Returns (L, ok)."""
    nb, n, _ = M.shape
    dtype = M.dtype
    L = np.zeros_like(M)
    ok = np.ones(nb, dtype=bool)
    for j in range(n):
        d = M[:, j, j].copy()
        for k in range(j):
            d = d - L[:, j, k] * L[:, j, k]
        ok &= d > 0
        ljj = np.sqrt(np.where(d > 0, d, dtype.type(np.nan)))
        L[:, j, j] = ljj
        for i in range(j + 1, n):
            s = M[:, i, j].copy()
            for k in range(j):
                s = s - L[:, i, k] * L[:, j, k]
            L[:, i, j] = s / ljj
    return L, ok


def chol_solve(L, R):
    """Solve (L L^T) X = R for R [B,n,m] (torch.cholesky_solve semantics)."""
    nb, n, m = R.shape
    Y = np.empty_like(R)
    for i in range(n):
        s = R[:, i, :].copy()
        for k in range(i):
            s = s - L[:, i, k, None] * Y[:, k, :]
        Y[:, i, :] = s / L[:, i, i, None]
    Xs = np.empty_like(R)
    for i in reversed(range(n)):
        s = Y[:, i, :].copy()
        for k in range(i + 1, n):
            s = s - L[:, k, i, None] * Xs[:, k, :]
        Xs[:, i, :] = s / L[:, i, i, None]
    return Xs


def _mT(a):
    return np.swapaxes(a, -1, -2)


def robust_gain_solve(Q_uu_reg, Q_ux, q_u, batch_fallback=False):
    """_robust_solve (controller.py:728-797): K = -Q^-1 Q_ux, k = -Q^-1 q_u by
    Cholesky; where the Cholesky fails, the reference falls back to an SVD
    inverse with singular values floored at S.max()/1e12. Under torch.vmap the
    reference's fallback is taken by the whole batch at that time step when
    any element fails; here it is taken per failing element (for the others
    the SVD and Cholesky solves agree to rounding times the condition number).
    A non-finite Q_uu (where the reference's SVD raises) gives NaN gains.
    Returns (K, k, fallback_used[B])."""
    L, ok = chol4(Q_uu_reg)
    K = -chol_solve(L, Q_ux)
    k = -chol_solve(L, q_u[..., None])[..., 0]
    bad = ~ok
    if batch_fallback and bad.any():
        bad = np.ones_like(bad)
    nonfinite = bad & ~np.isfinite(Q_uu_reg).all(axis=(-1, -2))
    if nonfinite.any():
        K[nonfinite] = np.nan
        k[nonfinite] = np.nan
        bad = bad & ~nonfinite
    if bad.any():
        Ub, S, Vh = np.linalg.svd(Q_uu_reg[bad])
        floor = S.max(axis=-1, keepdims=True) / Q_uu_reg.dtype.type(1e12)
        S_reg = np.where(S > floor, S, floor)
        Q_inv = _mT(Vh) @ (np.eye(S.shape[-1], dtype=S.dtype)[None] / S_reg[:, None, :]) @ _mT(Ub)
        K[bad] = -(Q_inv @ Q_ux[bad])
        k[bad] = -(Q_inv @ q_u[bad][..., None])[..., 0]
    return K, k, bad | nonfinite


# --------------------------------------------------------------------------
# Forward Riccati (controller.py:633-726, python-loop branch)
# --------------------------------------------------------------------------

def riccati(A, Bm, l_x, l_u, l_xx, l_xu, l_uu, l_xN, l_xxN, reg, batch_fallback=False):
    """backward_lqr (controller.py:697-726), batched over B.

    Q_uu carries reg*I once; the gain solve adds reg*I a second time
    (controller.py:706, :711); V, v use the once-regularised Q_uu.
    Returns K [B,T,nu,nx], k [B,T,nu], and a per-element flag set where a
    Cholesky failed and the SVD fallback was used.
    """
    dtype = A.dtype
    nb, T, nx = A.shape[:3]
    nu = Bm.shape[-1]
    I_nu = np.eye(nu, dtype=dtype)[None] * dtype.type(reg)
    V = l_xxN.copy()
    v = l_xN.copy()
    K = np.empty((nb, T, nu, nx), dtype=dtype)
    k = np.empty((nb, T, nu), dtype=dtype)
    chol_fail = np.zeros(nb, dtype=bool)
    for t in reversed(range(T)):
        At, Bt = A[:, t], Bm[:, t]
        AtT = _mT(At)
        Q_xx = l_xx[:, t] + (AtT @ V) @ At
        Q_xu = l_xu[:, t] + (AtT @ V) @ Bt
        Q_ux = _mT(Q_xu)
        Q_uu = l_uu[:, t] + (_mT(Bt) @ V) @ Bt + I_nu
        q_x = l_x[:, t] + (AtT @ v[..., None])[..., 0]
        q_u = l_u[:, t] + (_mT(Bt) @ v[..., None])[..., 0]
        Q_uu_reg = Q_uu + dtype.type(reg) * np.eye(nu, dtype=dtype)[None]
        Kt, kt, fb = robust_gain_solve(Q_uu_reg, Q_ux, q_u, batch_fallback)
        chol_fail |= fb
        K[:, t] = Kt
        k[:, t] = kt
        KtT = _mT(Kt)
        V = Q_xx + (KtT @ Q_uu) @ Kt + KtT @ Q_ux + Q_xu @ Kt
        v = (q_x + ((KtT @ Q_uu) @ kt[..., None])[..., 0] + (KtT @ q_u[..., None])[..., 0]
             + (Q_xu @ kt[..., None])[..., 0])
    return K, k, chol_fail


# --------------------------------------------------------------------------
# Grid line search (controller.py:437-533)
# --------------------------------------------------------------------------

def line_search(x0, Xn, Un, K, k, x_ref, u_ref, C, c, C_f, c_f, u_min, u_max,
                alphas, dt, model=None):
    """evaluate_alphas_batch_optimized (controller.py:437-533).

    u_t = U_t + a*k_t + a*(K_t (x_t - X_t)), clamped by max(., u_min) then
    min(., u_max) (controller.py:486-490). Returns candidates
    Xc [B,nA,T+1,nx], Uc [B,nA,T,nu], costs [B,nA].
    """
    model = model or DRONE10
    NX, NU = model.nx, model.nu
    dtype = x0.dtype
    nb = x0.shape[0]
    T = Un.shape[1]
    na = len(alphas)
    al = np.asarray(alphas, dtype=dtype)
    Xc = np.empty((nb, na, T + 1, NX), dtype=dtype)
    Uc = np.empty((nb, na, T, NU), dtype=dtype)
    x = np.repeat(x0[:, None, :], na, axis=1)
    Xc[:, :, 0] = x
    a = al[None, :, None]
    for t in range(T):
        dx = x - Xn[:, None, t]
        Kdx = np.einsum("bji,bai->baj", K[:, t], dx).astype(dtype)
        du = a * k[:, None, t] + a * Kdx
        u = Un[:, None, t] + du
        if u_min is not None:
            u = np.where(np.isnan(u), u, np.maximum(u, u_min))
        if u_max is not None:
            u = np.where(np.isnan(u), u, np.minimum(u, u_max))
        Uc[:, :, t] = u
        x = model.step(x.reshape(-1, NX), u.reshape(-1, NU), dt).reshape(nb, na, NX)
        Xc[:, :, t + 1] = x
    rep = lambda arr: np.repeat(arr, na, axis=0)
    costs = objective(Xc.reshape(nb * na, T + 1, NX), Uc.reshape(nb * na, T, NU),
                      rep(x_ref), rep(u_ref), rep(C), rep(c), rep(C_f), rep(c_f))
    return Xc, Uc, costs.reshape(nb, na)


def argmin_nan_first(costs):
    """torch.argmin semantics (controller.py:382): first NaN, else first min."""
    isn = np.isnan(costs)
    idx = np.argmin(np.where(isn, np.inf, costs), axis=1)
    any_nan = isn.any(axis=1)
    return np.where(any_nan, np.argmax(isn, axis=1), idx)


def tight_mask(U, u_min, u_max, atol=1e-7, rtol=1e-5):
    """_compute_tight_mask (controller.py:997-1003), torch.isclose semantics:
    a == b or |a - b| <= atol + rtol*|b| (evaluated in the input dtype)."""
    dtype = U.dtype
    m = np.zeros(U.shape, dtype=bool)
    for bnd in (u_min, u_max):
        if bnd is None:
            continue
        b = np.broadcast_to(np.asarray(bnd, dtype=dtype), U.shape)
        err = np.abs(U - b)
        allowed = dtype.type(atol) + np.abs(dtype.type(rtol) * b)
        m |= (U == b) | (np.isfinite(err) & (err <= allowed))
    return m


# --------------------------------------------------------------------------
# Solve (controller.py:303-435)
# --------------------------------------------------------------------------

def solve(x0, U_init, C, c, C_f=None, c_f=None, x_ref=None, u_ref=None,
          u_min=None, u_max=None, dt=0.05, max_iter=10, reg=1e-6,
          converge_tol=1e-6, alphas=DEFAULT_ALPHAS, forced=None,
          dtype=np.float32, reference_batch=False, model=None):
    """DifferentiableMPCController.solve_step (controller.py:303-435).

    Inputs are [B,...] arrays (C_f, c_f, x_ref, u_ref default to zeros, as on
    the FastMPC surface). ``reference_batch=True`` reproduces the reference's
    batch coupling for triage: every element (rejected ones included) runs
    every iteration, and a Cholesky failure anywhere at a time step switches
    the whole batch to the SVD solve (controller.py:745-760 under vmap). Returns a dict with X, U, trace, best_cost, iters
    (iterations each element ran), converged (the reference's global flag),
    tight (tight mask at the final U) and chol_fail. ``model`` is the
    dynamics (default: the reference's 10-state CTBR quadrotor).
    """
    model = model or DRONE10
    NX, NU = model.nx, model.nu
    N = NX + NU
    dtype = np.dtype(dtype)
    x0 = _f(x0, dtype)
    nb = x0.shape[0]
    U = _f(U_init, dtype).copy()
    T = U.shape[1]
    C = _f(C, dtype)
    c = _f(c, dtype)
    C_f = np.zeros((nb, N, N), dtype) if C_f is None else _f(C_f, dtype)
    c_f = np.zeros((nb, N), dtype) if c_f is None else _f(c_f, dtype)
    x_ref = np.zeros((nb, T + 1, NX), dtype) if x_ref is None else _f(x_ref, dtype)
    u_ref = np.zeros((nb, T, NU), dtype) if u_ref is None else _f(u_ref, dtype)
    u_min = None if u_min is None else _f(u_min, dtype)
    u_max = None if u_max is None else _f(u_max, dtype)

    X = rollout(x0, U, dt, model)
    best = objective(X, U, x_ref, u_ref, C, c, C_f, c_f)
    active = np.ones(nb, dtype=bool)
    trace = np.full((nb, max_iter), NOT_RUN, dtype=np.int8)
    iters = np.zeros(nb, dtype=np.int32)
    stall_iter = np.full(nb, max_iter, dtype=np.int64)
    stall_gap = np.zeros(nb, dtype=np.float64)
    chol_fail = np.zeros(nb, dtype=bool)
    for i in range(max_iter):
        if forced is not None:
            active &= np.asarray(forced)[:, i] != NOT_RUN
        if not active.any():
            break
        ids = np.nonzero(active)[0]
        if reference_batch:
            ids = np.arange(nb) if forced is None else np.nonzero(np.asarray(forced)[:, i] != NOT_RUN)[0]
            if len(ids) == 0:
                break
        sub = lambda arr: arr[ids]
        l_x, l_u, l_xx, l_xu, l_uu, l_xN, l_xxN = quadraticize(
            sub(X), sub(U), sub(x_ref), sub(u_ref), sub(C), sub(c), sub(C_f), sub(c_f))
        A, Bm = linearize(sub(X), sub(U), dt, model)
        K, k, cf = riccati(A, Bm, l_x, l_u, l_xx, l_xu, l_uu, l_xN, l_xxN, reg,
                           batch_fallback=reference_batch)
        chol_fail[ids] |= cf
        Xc, Uc, costs = line_search(sub(x0), sub(X), sub(U), K, k, sub(x_ref), sub(u_ref),
                                    sub(C), sub(c), sub(C_f), sub(c_f), u_min, u_max,
                                    alphas, dt, model)
        j = argmin_nan_first(costs)
        new = costs[np.arange(len(ids)), j]
        if forced is None:
            improved = new < best[ids]
            stop = ~improved
        else:
            f = np.asarray(forced)[ids, i].astype(np.int64)
            improved = f >= 0
            j = np.where(improved, f, j)
            new = costs[np.arange(len(ids)), j]
            stop = np.zeros(len(ids), dtype=bool)
        iters[ids] += 1
        trace[ids, i] = np.where(improved, j, -(j + 1)).astype(np.int8)
        acc = ids[improved]
        rej = ids[~improved]
        X[acc] = Xc[improved, j[improved]]
        U[acc] = Uc[improved, j[improved]]
        first_rej = rej[stall_iter[rej] == max_iter]
        stall_iter[first_rej] = i
        stall_gap[first_rej] = np.abs(new[np.isin(ids, first_rej)].astype(np.float64)
                                      - best[first_rej].astype(np.float64))
        best[acc] = new[improved]
        active[ids[stop]] = False
    converged = global_converged_flag(stall_iter, stall_gap, max_iter, converge_tol,
                                      np.isfinite(X).all() and np.isfinite(U).all())
    return dict(X=X, U=U, trace=trace, best_cost=best, iters=iters, converged=converged,
                tight=tight_mask(U, u_min, u_max), chol_fail=chol_fail,
                stall_iter=stall_iter, stall_gap=stall_gap)


def global_converged_flag(stall_iter, stall_gap, max_iter, converge_tol, all_finite):
    """The reference's `converged` after solve_step (controller.py:396-423),
    reconstructed from per-element stalls: the first iteration with no
    improvement anywhere is s = max(stall_iter); from there every iteration
    recomputes the same costs, so the loop breaks at s if the largest gap is
    below converge_tol, else at s+2 (third consecutive stall) if that is still
    inside max_iter. A loop that runs out of iterations reports convergence
    iff X and U are finite."""
    s = int(np.max(stall_iter)) if len(stall_iter) else 0
    if s < max_iter:
        gap = float(np.max(stall_gap)) if len(stall_gap) else 0.0
        if (not np.isnan(gap) and gap < converge_tol) or s + 2 <= max_iter - 1:
            return True
    return bool(all_finite)


# --------------------------------------------------------------------------
# Implicit-differentiation backward (controller.py:68-133, 1006-1131)
# --------------------------------------------------------------------------

def zero_constrained_lqr(A, Bm, H_xx, H_uu, H_xu, grad_x, grad_u, tight,
                         grad_x_final, H_xx_final, reg):
    """_zero_constrained_lqr (controller.py:1006-1131).

    Masked adjoint Riccati: tight rows/cols of Q_uu zeroed with +1 on their
    diagonal plus a (1e-8*reg)*I ridge; Q_ux tight rows and q_u tight entries
    zeroed; V and v are then updated with the UNMASKED Q_uu, Q_ux, q_u.
    Sweep: dU = K dX + k, dX_{t+1} = A dX + B dU, dX_0 = 0.
    Returns dX [B,T+1,nx], dU [B,T,nu], v0 [B,nx], K, k.
    """
    dtype = A.dtype
    nb, T, NX = A.shape[:3]
    NU = Bm.shape[-1]
    V = H_xx_final.copy()
    v = grad_x_final.copy()
    eye = np.eye(NU, dtype=dtype)[None]
    I_nu = eye * dtype.type(reg)
    K = np.empty((nb, T, NU, NX), dtype=dtype)
    k = np.empty((nb, T, NU), dtype=dtype)
    for t in reversed(range(T)):
        At, Bt = A[:, t], Bm[:, t]
        V_A = V @ At
        V_B = V @ Bt
        Q_xx = H_xx[:, t] + _mT(At) @ V_A
        Q_xu = H_xu[:, t] + _mT(At) @ V_B
        Q_ux = _mT(Q_xu)
        Q_uu = H_uu[:, t] + _mT(Bt) @ V_B + I_nu
        q_x = grad_x[:, t] + (_mT(At) @ v[..., None])[..., 0]
        q_u = grad_u[:, t] + (_mT(Bt) @ v[..., None])[..., 0]
        m = tight[:, t].astype(bool)
        mb = m[:, :, None] | m[:, None, :]
        Q_uu_m = np.where(mb, dtype.type(0), Q_uu) + m[:, None, :] * eye
        Q_ux_m = np.where(m[:, :, None], dtype.type(0), Q_ux)
        q_u_m = np.where(m, dtype.type(0), q_u)
        Q_uu_reg = Q_uu_m + dtype.type(1e-8) * I_nu
        L, ok = chol4(Q_uu_reg)
        Kt = -chol_solve(L, Q_ux_m)
        kt = -chol_solve(L, q_u_m[..., None])[..., 0]
        if not ok.all():
            # controller.py:1089-1092: a failed Cholesky falls back to an LU
            # solve (taken per element here; the reference takes it batch-wide).
            bad = ~ok
            Kt[bad] = -np.linalg.solve(Q_uu_reg[bad], Q_ux_m[bad])
            kt[bad] = -np.linalg.solve(Q_uu_reg[bad], q_u_m[bad][..., None])[..., 0]
        K[:, t] = Kt
        k[:, t] = kt
        KtT = _mT(Kt)
        V = Q_xx + KtT @ (Q_uu @ Kt) + KtT @ Q_ux + Q_xu @ Kt
        q_u_aug = (Q_uu @ kt[..., None])[..., 0] + q_u
        v = q_x + (KtT @ q_u_aug[..., None])[..., 0] + (Q_xu @ kt[..., None])[..., 0]
    dX = np.zeros((nb, T + 1, NX), dtype=dtype)
    dU = np.zeros((nb, T, NU), dtype=dtype)
    for t in range(T):
        dx = dX[:, t]
        du = (K[:, t] @ dx[..., None])[..., 0] + k[:, t]
        dU[:, t] = du
        dX[:, t + 1] = (A[:, t] @ dx[..., None])[..., 0] + (Bm[:, t] @ du[..., None])[..., 0]
    return dX, dU, v, K, k


def backward(X, U, C, C_f, x_ref, u_ref, tight, grad_X, grad_U, dt, reg,
             dtype=np.float32, model=None):
    """ILQRSolve.backward (controller.py:68-133) at a solved (X, U).

    grad_C = -1/2 (dtau (x) z + z (x) dtau) with z = [X_t; U_t] (not tau);
    grad_c = -dtau; grad_x0 = -v0; grad_xref[:T] = dX[:T], grad_xref[T] = 0;
    grad_uref = dU; grad_C_final xx block = -1/2 (dX_T (x) e + e (x) dX_T),
    e = X_T - x_ref_T; grad_c_final[:nx] = -dX_T.
    """
    model = model or DRONE10
    NX, NU = model.nx, model.nu
    N = NX + NU
    dtype = np.dtype(dtype)
    X = _f(X, dtype)
    U = _f(U, dtype)
    nb, T = U.shape[:2]
    C = _f(C, dtype)
    C_f = np.zeros((nb, N, N), dtype) if C_f is None else _f(C_f, dtype)
    x_ref = np.zeros((nb, T + 1, NX), dtype) if x_ref is None else _f(x_ref, dtype)
    u_ref = np.zeros((nb, T, NU), dtype) if u_ref is None else _f(u_ref, dtype)
    gX = _f(grad_X, dtype)
    gU = _f(grad_U, dtype)
    A, Bm = linearize(X, U, dt, model)
    H_xx, H_xu, H_uu = C[..., :NX, :NX], C[..., :NX, NX:], C[..., NX:, NX:]
    dX, dU, v0, K, k = zero_constrained_lqr(
        A, Bm, H_xx, H_uu, H_xu, -gX[:, :-1], -gU, tight, -gX[:, -1],
        C_f[:, :NX, :NX], reg)
    half = dtype.type(0.5)
    outer = lambda a, b: a[..., :, None] * b[..., None, :]
    Xs = X[:, :-1]
    grad_C = np.zeros((nb, T, N, N), dtype=dtype)
    grad_C[:, :, :NX, :NX] = -half * (outer(dX[:, :-1], Xs) + outer(Xs, dX[:, :-1]))
    grad_C[:, :, NX:, NX:] = -half * (outer(dU, U) + outer(U, dU))
    d_xu = -half * (outer(dX[:, :-1], U) + outer(Xs, dU))
    grad_C[:, :, :NX, NX:] = d_xu
    grad_C[:, :, NX:, :NX] = _mT(d_xu)
    grad_c = -np.concatenate([dX[:, :-1], dU], axis=-1)
    grad_xref = np.zeros_like(x_ref)
    grad_xref[:, :T] = -grad_c[..., :NX]
    grad_uref = -grad_c[..., NX:]
    err = X[:, -1] - x_ref[:, -1]
    dxN = dX[:, -1]
    grad_C_f = np.zeros((nb, N, N), dtype=dtype)
    grad_C_f[:, :NX, :NX] = -half * (outer(dxN, err) + outer(err, dxN))
    grad_c_f = np.zeros((nb, N), dtype=dtype)
    grad_c_f[:, :NX] = -dxN
    return dict(grad_x0=-v0, grad_C=grad_C, grad_c=grad_c, grad_C_final=grad_C_f,
                grad_c_final=grad_c_f, grad_xref=grad_xref, grad_uref=grad_uref,
                dX=dX, dU=dU, K=K, k=k)


def _sigmoid_slices(T):
    """(offset into x_q, length-T index) of each tau entry's block.
    _build_cost_tensors (training_modules/mlp_mpc_policy_diffmpc.py:204-216)
    slices x_q / x_p into blocks of T steps: p (3), q (4), v (3), w (3),
    thrust (1); the diagonal and c list them in tau order p, q, v, thrust, w
    (:226-243)."""
    t = np.arange(T)
    idx = np.empty((T, N), dtype=np.int64)
    for i in range(3):
        idx[:, i] = 3 * t + i
    for i in range(4):
        idx[:, 3 + i] = 3 * T + 4 * t + i
    for i in range(3):
        idx[:, 7 + i] = 7 * T + 3 * t + i
    idx[:, 10] = 13 * T + t
    for i in range(3):
        idx[:, 11 + i] = 10 * T + 3 * t + i
    return idx


def sigmoid_costs(sc, T, eps=0.1, range_q=100000.0, range_p=100000.0, range_pt=None, mass=MASS):
    """C [B,T,14,14] (diagonal) and c [B,T,14] from the policy's sigmoid output
    sc [B, 28 T], in float32 with the reference's operation order
    (_build_cost_tensors, mlp_mpc_policy_diffmpc.py:194-247):
    x_q = sc[:, :14T] * range_q + eps; x_p = sc[:, 14T:];
    c = (x_p - 0.5) * range_p, thrust entry c = -(x_p * range_pt + eps)
    with range_pt = range_q * mass * 9.806 (a Python float, rounded to fp32)."""
    f32 = np.float32
    sc = np.asarray(sc, dtype=f32)
    nb = sc.shape[0]
    rpt = f32(range_q * mass * 9.806 if range_pt is None else range_pt)
    x_q = sc[:, :14 * T] * f32(range_q) + f32(eps)
    x_p = sc[:, 14 * T:]
    idx = _sigmoid_slices(T)
    diag = x_q[:, idx]                                   # [B, T, 14]
    xp = x_p[:, idx]
    c = (xp - f32(0.5)) * f32(range_p)
    c[..., 10] = -(xp[..., 10] * rpt + f32(eps))
    C = np.zeros((nb, T, N, N), dtype=f32)
    ii = np.arange(N)
    C[:, :, ii, ii] = diag
    return C, c.astype(f32)


def sigmoid_cost_grad(grad_C, grad_c, T, range_q=100000.0, range_p=100000.0, range_pt=None, mass=MASS):
    """Gradient of the sigmoid output through sigmoid_costs (the chain rule
    torch's autograd applies to _build_cost_tensors): the diagonal of grad_C
    times range_q, grad_c times range_p, and for the thrust entry
    (-grad_c) * range_pt."""
    f32 = np.float32
    rpt = f32(range_q * mass * 9.806 if range_pt is None else range_pt)
    grad_C = np.asarray(grad_C, dtype=f32)
    grad_c = np.asarray(grad_c, dtype=f32)
    nb = grad_C.shape[0]
    idx = _sigmoid_slices(T)
    ii = np.arange(N)
    g = np.zeros((nb, 28 * T), dtype=f32)
    g[:, idx] = grad_C[:, :, ii, ii] * f32(range_q)
    gp = grad_c * f32(range_p)
    gp[..., 10] = (-grad_c[..., 10]) * rpt
    g[:, 14 * T + idx] = gp
    return g


def _solve4_pivot(A, b):
    """Gaussian elimination with partial pivoting on one 4x4 system (float32),
    pivots of magnitude below 1e-10 replaced by +-1e-10, as the reference's
    PNQP step (differentialMPCPerformance/cpp/pnqp_kernel.cuh:15-54)."""
    f32 = np.float32
    A = A.astype(f32).copy()
    b = b.astype(f32).copy()
    for k in range(4):
        r = k + int(np.argmax(np.abs(A[k:, k])))
        if np.abs(A[r, k]) > np.abs(A[k, k]) and r != k:
            A[[k, r]] = A[[r, k]]
            b[[k, r]] = b[[r, k]]
        piv = A[k, k]
        if abs(piv) < f32(1e-10):
            piv = f32(-1e-10) if piv < 0 else f32(1e-10)
        for i in range(k + 1, 4):
            f = f32(A[i, k] / piv)
            for j in range(k + 1, 4):
                A[i, j] = f32(A[i, j] - f32(f * A[k, j]))
            b[i] = f32(b[i] - f32(f * b[k]))
            A[i, k] = 0
    x = np.zeros(4, f32)
    for i in range(3, -1, -1):
        s_ = b[i]
        for j in range(i + 1, 4):
            s_ = f32(s_ - f32(A[i, j] * x[j]))
        x[i] = f32(s_ / A[i, i])
    return x


def pnqp4(H, q, lower, upper, x_init=None):
    """Projected-Newton box QP min 1/2 x^T H x + q^T x, lower <= x <= upper, for
    [N,4] problems (the reference's PNQP-4, pnqp_kernel.cuh:91-208, with
    mpc.pytorch.pnqp's constants: ridge 1e-11, Armijo gamma 0.1, decay 0.1,
    step tolerance 1e-4; per problem: at most 10 Newton steps, 10 Armijo
    trials, a bound counts as active within 1e-8). A zero x_init starts from the
    unconstrained solution. Returns (x*, free_mask) in float32."""
    f32 = np.float32
    H = np.asarray(H, f32)
    q = np.asarray(q, f32)
    lo = np.asarray(lower, f32)
    hi = np.asarray(upper, f32)
    n = H.shape[0]
    X = np.zeros((n, 4), f32)
    F = np.zeros((n, 4), f32)
    eps = f32(1e-8)
    obj = lambda h, qq, x: f32(f32(0.5) * f32(x @ (h @ x))) + f32(qq @ x)
    for b in range(n):
        x = np.zeros(4, f32) if x_init is None else np.asarray(x_init[b], f32).copy()
        if not np.any(x != 0):
            x = _solve4_pivot(H[b], -q[b])
        x = np.minimum(np.maximum(x, lo[b]), hi[b])
        for _ in range(10):
            g = (H[b] @ x + q[b]).astype(f32)
            clamped = ((x <= lo[b] + eps) & (g > 0)) | ((x >= hi[b] - eps) & (g < 0))
            fr = (~clamped).astype(f32)
            Hm = (H[b] * fr[:, None] * fr[None, :]).astype(f32) + np.eye(4, dtype=f32) * f32(1e-11)
            dx = _solve4_pivot(Hm, -g * fr)
            if float(dx @ dx) < 1e-8:
                break
            ox = obj(H[b], q[b], x)
            alpha = f32(1.0)
            for _ls in range(10):
                mx = np.minimum(np.maximum(x + alpha * dx, lo[b]), hi[b]).astype(f32)
                om = obj(H[b], q[b], mx)
                den = f32(g @ (x - mx))
                arm = (ox - om) / (den if abs(den) > 1e-12 else f32(1e-12))
                if arm > 0.1:
                    break
                alpha = f32(alpha * f32(0.1))
            x = mx
        g = (H[b] @ x + q[b]).astype(f32)
        clamped = ((x <= lo[b] + eps) & (g > 0)) | ((x >= hi[b] - eps) & (g < 0))
        X[b] = x
        F[b] = (~clamped).astype(f32)
    return X, F


__all__ = [
    "NX", "NU", "N", "MASS", "GRAV_Z", "NOT_RUN", "DEFAULT_ALPHAS", "Model", "DRONE10",
    "drone_step", "drone_jacobian", "rollout", "linearize", "objective",
    "quadraticize", "chol4", "chol_solve", "riccati", "line_search",
    "argmin_nan_first", "tight_mask", "solve", "global_converged_flag",
    "zero_constrained_lqr", "backward", "sigmoid_costs", "sigmoid_cost_grad", "pnqp4",
]
