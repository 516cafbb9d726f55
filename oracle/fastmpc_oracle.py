"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the reference FastMPC
extension's CUDA build (differentialMPCPerformance/cpp, compiled with the
fused forward and backward kernels and the PNQP-aware Riccati pass, as
drone_ilqr.py:140-158 selects them).

This is the "FastMPC numerics" mode: the numerics that the reference's own
`mpc_compat.FastMPC` runs, as opposed to the DiffMPC numerics of
diffmpc_oracle.py. Differences from DiffMPC, each restated below with its
reference lines:

- the model step renormalises the quaternion, and the Jacobian is the Euler
  Jacobian of the continuous dynamics with the correct sign on every entry
  (drone_kernels.cu:64-190, forward_pass_kernel.cu:66-115);
- Q_uu carries the regulariser once; gains come from a pivoted LU;
  V = Q_xx + Q_xu K and v = q_x + Q_xu k (backward_pass_kernel.cu:787-1047);
- with control bounds, each Riccati step first solves the box QP of the step
  at dx = 0 with PNQP-4; its free mask zeroes the clamped rows and columns of
  Q_uu (1e-11 ridge), the clamped columns of Q_xu and entries of q_u, and the
  clamped entries of k are the PNQP optimum (same lines);
- the line search tries alpha in (1, 0.5, 0.25, 0.1) with
  u = U + alpha k + K dx, K not scaled (drone_ilqr_ext.cpp:736,
  forward_pass_kernel.cu:160-189);
- convergence is one flag for the whole batch, read every fourth iteration
  and at the last: stop when max_b |best_b - new_b| < converge_tol
  (drone_ilqr_ext.cpp:1029-1049);
- the tight mask is the free mask of the last Riccati pass run, and the
  backward linearises where that pass did (drone_ilqr_ext.cpp:1052-1063);
- the backward is the masked adjoint Riccati of backward_pass_kernel.cu:
  617-745 and the assembly of :1092-1256 (grad_x_ref[T] = dX_T, tau built
  from X - x_ref).

The reference extension as a whole is not built here (it needs libtorch); its
CUDA kernels are, from their own sources (oracle/build_fastmpc_ref.py), and the
GPU tests re-drive them (oracle/fastmpc_ref_cuda.py). Arithmetic is fp32
with the reference kernels' operation order: sums in index order, each product
rounded, divisions exact. (The reference compiles with --use_fast_math, which
contracts products into fused multiply-adds and makes division approximate,
as the B200 kernels do; that rounding is not restated, and the parity bars
absorb it.) Pinned pieces: pnqp4 against mpc.pytorch's pnqp (golden
vectors), the Jacobian against central differences of the continuous
dynamics, and the Riccati pass, line search and adjoint against the closed
form of linear-quadratic problems (tests/test_oracle_fastmpc.py).

Decision traces follow diffmpc_oracle: trace[b, i] = j (accepted candidate
j), -(j + 1) (rejected, argmin j), -128 (iteration not run). A replay also
fixes the iteration at which the batch stopped.
"""

from __future__ import annotations

import numpy as np

from .diffmpc_oracle import NOT_RUN, pnqp4

F32 = np.float32
NX, NU, N = 10, 4, 14
MASS = F32(0.752)          # drone_kernels.cu:12
G_VAL = F32(-9.8066)       # drone_kernels.cu:13
FM_ALPHAS = (1.0, 0.5, 0.25, 0.1)   # drone_ilqr_ext.cpp:736
CHECK_PERIOD = 4                    # drone_ilqr_ext.cpp:763


def _f(a):
    return np.asarray(a, dtype=F32)


# --------------------------------------------------------------------------
# Model: the extension's CUDA step and Jacobian
# --------------------------------------------------------------------------

def _exp_map(wx, wy, wz, dt):
    """forward_pass_kernel.cu:26-39 (drone_kernels.cu:31-45 rounds the same:
    scaling by 0.5 is exact)."""
    w_norm = np.sqrt(wx * wx + wy * wy + wz * wz) + F32(1e-8)
    half = w_norm * (F32(dt) * F32(0.5))
    s = np.sin(half)
    c = np.cos(half)
    inv = F32(1.0) / w_norm
    return c, wx * inv * s, wy * inv * s, wz * inv * s


def _quat_step(qw, qx, qy, qz, wx, wy, wz, dt):
    """q (x) exp_map(w, dt), renormalised (forward_pass_kernel.cu:86-99)."""
    ew, ex, ey, ez = _exp_map(wx, wy, wz, dt)
    nw = qw * ew - qx * ex - qy * ey - qz * ez
    nx = qw * ex + qx * ew + qy * ez - qz * ey
    ny = qw * ey - qx * ez + qy * ew + qz * ex
    nz = qw * ez + qx * ey - qy * ex + qz * ew
    qn = np.sqrt(nw * nw + nx * nx + ny * ny + nz * nz) + F32(1e-8)
    return nw / qn, nx / qn, ny / qn, nz / qn


def fm_step(x, u, dt):
    """Line-search step (forward_pass_kernel.cu:66-115): thrust rotated by the
    cross-product form of q v q^-1 with the old quaternion. x [..,10], u [..,4]."""
    x = _f(x)
    u = _f(u)
    dt = F32(dt)
    px, py, pz, qw, qx, qy, qz, vx, vy, vz = (x[..., i] for i in range(10))
    fc, wx, wy, wz = (u[..., i] for i in range(4))
    zero = F32(0.0)
    nq = _quat_step(qw, qx, qy, qz, wx, wy, wz, dt)
    tx = qy * fc - qz * zero
    ty = qz * zero - qx * fc
    tz = qx * zero - qy * zero
    ttx = qy * tz - qz * ty
    tty = qz * tx - qx * tz
    ttz = qx * ty - qy * tx
    ax = (zero + F32(2.0) * (qw * tx + ttx)) / MASS
    ay = (zero + F32(2.0) * (qw * ty + tty)) / MASS
    az = (fc + F32(2.0) * (qw * tz + ttz)) / MASS + G_VAL
    return np.stack([px + vx * dt, py + vy * dt, pz + vz * dt, *nq,
                     vx + ax * dt, vy + ay * dt, vz + az * dt], axis=-1).astype(F32)


def fm_rollout_step(x, u, dt):
    """Initial-rollout step (drone_kernels.cu:195-250): the same model with the
    rotation-matrix form of q v q^-1."""
    x = _f(x)
    u = _f(u)
    dt = F32(dt)
    px, py, pz, qw, qx, qy, qz, vx, vy, vz = (x[..., i] for i in range(10))
    fc, wx, wy, wz = (u[..., i] for i in range(4))
    zero = F32(0.0)
    two = F32(2.0)
    nq = _quat_step(qw, qx, qy, qz, wx, wy, wz, dt)
    q00, q11, q22, q33 = qw * qw, qx * qx, qy * qy, qz * qz
    q01, q02, q03 = qw * qx, qw * qy, qw * qz
    q12, q13, q23 = qx * qy, qx * qz, qy * qz
    rx = (q00 + q11 - q22 - q33) * zero + two * (q12 - q03) * zero + two * (q13 + q02) * fc
    ry = two * (q12 + q03) * zero + (q00 - q11 + q22 - q33) * zero + two * (q23 - q01) * fc
    rz = two * (q13 - q02) * zero + two * (q23 + q01) * zero + (q00 - q11 - q22 + q33) * fc
    return np.stack([px + vx * dt, py + vy * dt, pz + vz * dt, *nq,
                     vx + (rx / MASS) * dt, vy + (ry / MASS) * dt, vz + (rz / MASS + G_VAL) * dt],
                    axis=-1).astype(F32)


def fm_jacobian(x, u, dt):
    """A [..,10,10], B [..,10,4]: the Euler Jacobian I + dt J of the continuous
    dynamics (drone_kernels.cu:124-190)."""
    x = _f(x)
    u = _f(u)
    dt = F32(dt)
    qw, qx, qy, qz = (x[..., i] for i in range(3, 7))
    fc, wx, wy, wz = (u[..., i] for i in range(4))
    sh = x.shape[:-1]
    A = np.zeros(sh + (10, 10), F32)
    B = np.zeros(sh + (10, 4), F32)
    for i in range(10):
        A[..., i, i] = 1.0
    A[..., 0, 7] = dt
    A[..., 1, 8] = dt
    A[..., 2, 9] = dt
    h = F32(0.5) * dt
    zero = F32(0.0)
    A[..., 3, 4] = zero - h * wx
    A[..., 3, 5] = zero - h * wy
    A[..., 3, 6] = zero - h * wz
    A[..., 4, 3] = zero + h * wx
    A[..., 4, 5] = zero + h * wz
    A[..., 4, 6] = zero - h * wy
    A[..., 5, 3] = zero + h * wy
    A[..., 5, 4] = zero - h * wz
    A[..., 5, 6] = zero + h * wx
    A[..., 6, 3] = zero + h * wz
    A[..., 6, 4] = zero + h * wy
    A[..., 6, 5] = zero - h * wx
    mh = -h
    B[..., 3, 1] = mh * qx
    B[..., 3, 2] = mh * qy
    B[..., 3, 3] = mh * qz
    B[..., 4, 1] = h * qw
    B[..., 4, 2] = mh * qz
    B[..., 4, 3] = h * qy
    B[..., 5, 1] = h * qz
    B[..., 5, 2] = h * qw
    B[..., 5, 3] = mh * qx
    B[..., 6, 1] = mh * qy
    B[..., 6, 2] = h * qx
    B[..., 6, 3] = h * qw
    fcm = fc / MASS
    t2 = F32(2.0) * dt
    q0, q1, q2, q3 = qw * fcm, qx * fcm, qy * fcm, qz * fcm
    A[..., 7, 3], A[..., 7, 4], A[..., 7, 5], A[..., 7, 6] = t2 * q2, t2 * q3, t2 * q0, t2 * q1
    A[..., 8, 3], A[..., 8, 4], A[..., 8, 5], A[..., 8, 6] = -t2 * q1, -t2 * q0, t2 * q3, t2 * q2
    A[..., 9, 3], A[..., 9, 4], A[..., 9, 5], A[..., 9, 6] = t2 * q0, -t2 * q1, -t2 * q2, t2 * q3
    dtm = dt / MASS
    B[..., 7, 0] = F32(2.0) * (qx * qz + qw * qy) * dtm
    B[..., 8, 0] = F32(2.0) * (qy * qz - qw * qx) * dtm
    B[..., 9, 0] = (qw * qw - qx * qx - qy * qy + qz * qz) * dtm
    return A, B


def fm_rollout(x0, U, dt, step=None):
    """X [B,T+1,10] from x0 and (already clamped) U (drone_ilqr_ext.cpp:577-618)."""
    step = fm_rollout_step if step is None else step
    x0 = _f(x0)
    U = _f(U)
    B, T = U.shape[:2]
    X = np.empty((B, T + 1, x0.shape[-1]), F32)
    X[:, 0] = x0
    for t in range(T):
        X[:, t + 1] = step(X[:, t], U[:, t], dt)
    return X


# --------------------------------------------------------------------------
# Cost
# --------------------------------------------------------------------------

def _mv(M, z):
    """M [B,n,m] z [B,m] with a sequential sum over m (fp32)."""
    s = M[..., 0] * z[:, None, 0]
    for k in range(1, M.shape[-1]):
        s = s + M[..., k] * z[:, None, k]
    return s.astype(F32)


def _seqsum(a):
    """Sum over the last axis, first entry then the others in order (fp32)."""
    s = a[..., 0]
    for k in range(1, a.shape[-1]):
        s = s + a[..., k]
    return s.astype(F32)


def fm_cost(X, U, C, c, C_f, c_f, x_ref, u_ref, form="total"):
    """Total cost per element, sums in index order. form "total":
    compute_cost (drone_ilqr_ext.cpp:620-663), sum_t (0.5 (z^T C z) + z^T c),
    then + 0.5 z_N^T C_f z_N, then + z_N^T c_f; form "line_search": the
    candidate costs of :987-1001, which scale each product by 0.5 before
    summing and add the terminal term as one."""
    T = U.shape[1]
    total = np.zeros(X.shape[0], F32)
    for t in range(T):
        z = np.concatenate([X[:, t] - x_ref[:, t], U[:, t] - u_ref[:, t]], axis=-1).astype(F32)
        Cz = _mv(C[:, t], z)
        if form == "total":
            step = F32(0.5) * _seqsum(z * Cz) + _seqsum(z * c[:, t])
        else:
            step = _seqsum(F32(0.5) * (z * Cz)) + _seqsum(z * c[:, t])
        total = (total + step).astype(F32)
    zN = np.concatenate([X[:, T] - x_ref[:, T], np.zeros((X.shape[0], U.shape[-1]), F32)], axis=-1).astype(F32)
    CzN = _mv(C_f, zN)
    if form == "total":
        return ((total + F32(0.5) * _seqsum(zN * CzN)) + _seqsum(zN * c_f)).astype(F32)
    return (total + (_seqsum(F32(0.5) * (zN * CzN)) + _seqsum(zN * c_f))).astype(F32)


def fm_quadraticize(X, U, C, c, C_f, c_f, x_ref, u_ref):
    """l_xx, l_uu, l_xu are slices of C; l_x = l_xx e_x + l_xu e_u + c_x and
    l_u = l_xu^T e_x + l_uu e_u + c_u; l_xN = C_f[:nx,:nx] e_xN + c_f[:nx]
    (drone_ilqr_ext.cpp:797-823)."""
    nx = X.shape[-1]
    T = U.shape[1]
    ex = (X[:, :T] - x_ref[:, :T]).astype(F32)
    eu = (U - u_ref).astype(F32)
    lxx = C[:, :, :nx, :nx]
    luu = C[:, :, nx:, nx:]
    lxu = C[:, :, :nx, nx:]
    lx = np.empty(ex.shape, F32)
    lu = np.empty(eu.shape, F32)
    for t in range(T):
        lx[:, t] = (_mv(lxx[:, t], ex[:, t]) + _mv(lxu[:, t], eu[:, t]) + c[:, t, :nx]).astype(F32)
        lu[:, t] = (_mv(np.swapaxes(lxu[:, t], -1, -2), ex[:, t]) + _mv(luu[:, t], eu[:, t])
                    + c[:, t, nx:]).astype(F32)
    exN = (X[:, T] - x_ref[:, T]).astype(F32)
    lxxN = np.ascontiguousarray(C_f[:, :nx, :nx])
    lxN = (_mv(lxxN, exN) + c_f[:, :nx]).astype(F32)
    return lxx, luu, lxu, lx, lu, lxxN, lxN


# --------------------------------------------------------------------------
# 4x4 LU of the extension (backward_pass_kernel.cu:420-470)
# --------------------------------------------------------------------------

def lu_factor4(M):
    """In-place pivoted LU of [B,4,4]; a pivot below 1e-10 in magnitude is
    replaced by +-1e-10 for the multipliers only (the stored diagonal keeps
    its value). Returns (LU, piv)."""
    A = _f(M).copy()
    Bn = A.shape[0]
    piv = np.zeros((Bn, 4), np.int64)
    rows = np.arange(Bn)
    for k in range(4):
        mr = np.full(Bn, k)
        mv = np.abs(A[:, k, k])
        for i in range(k + 1, 4):
            v = np.abs(A[:, i, k])
            upd = v > mv
            mv = np.where(upd, v, mv)
            mr = np.where(upd, i, mr)
        piv[:, k] = mr
        rk = A[rows, k].copy()
        A[rows, k] = A[rows, mr]
        A[rows, mr] = rk
        p = A[:, k, k].copy()
        small = np.abs(p) < F32(1e-10)
        p = np.where(small, np.where(p < 0, F32(-1e-10), F32(1e-10)), p).astype(F32)
        for i in range(k + 1, 4):
            A[:, i, k] = A[:, i, k] / p
            for j in range(k + 1, 4):
                A[:, i, j] = A[:, i, j] - A[:, i, k] * A[:, k, j]
    return A, piv


def lu_solve4(LU, piv, b):
    """Solve with lu_factor4's factors; b [B,4] (backward_pass_kernel.cu:474-496)."""
    b = _f(b).copy()
    rows = np.arange(b.shape[0])
    for k in range(4):
        bk = b[rows, k].copy()
        b[rows, k] = b[rows, piv[:, k]]
        b[rows, piv[:, k]] = bk
    for k in range(4):
        for i in range(k + 1, 4):
            b[:, i] = b[:, i] - LU[:, i, k] * b[:, k]
    for i in range(3, -1, -1):
        s = b[:, i].copy()
        for j in range(i + 1, 4):
            s = s - LU[:, i, j] * b[:, j]
        b[:, i] = s / LU[:, i, i]
    return b


# --------------------------------------------------------------------------
# Riccati passes
# --------------------------------------------------------------------------

def _q_terms(V, v, A, B, lxx, luu, lxu, lx, lu, reg):
    """Q terms of one step (backward_pass_kernel.cu:871-934): sequential sums
    started from the cost term, reg added to Q_uu's diagonal once."""
    nx = A.shape[-1]
    nu = B.shape[-1]
    VA = np.zeros(A.shape, F32)
    VB = np.zeros(B.shape, F32)
    for k in range(nx):
        VA = VA + V[:, :, k, None] * A[:, None, k, :]
        VB = VB + V[:, :, k, None] * B[:, None, k, :]
    Qxx = lxx.astype(F32).copy()
    Qxu = lxu.astype(F32).copy()
    qx = lx.astype(F32).copy()
    Quu = luu.astype(F32).copy()
    qu = lu.astype(F32).copy()
    for k in range(nx):
        Qxx = Qxx + A[:, k, :, None] * VA[:, k, None, :]
        Qxu = Qxu + A[:, k, :, None] * VB[:, k, None, :]
        qx = qx + A[:, k, :] * v[:, k, None]
        Quu = Quu + B[:, k, :, None] * VB[:, k, None, :]
        qu = qu + B[:, k, :] * v[:, k, None]
    for i in range(nu):
        Quu[:, i, i] = Quu[:, i, i] + F32(reg)
    return Qxx, Qxu, Quu, qx, qu


def _apply_free_mask(Quu, Qxu, qu, fm):
    Quu = (Quu * (fm[:, :, None] * fm[:, None, :])).astype(F32)
    for i in range(Quu.shape[-1]):
        Quu[:, i, i] = np.where(fm[:, i] == 0, Quu[:, i, i] + F32(1e-11), Quu[:, i, i])
    return Quu, (Qxu * fm[:, None, :]).astype(F32), (qu * fm).astype(F32)


def _gains(Quu, Qxu, qu):
    LU, piv = lu_factor4(Quu)
    nx = Qxu.shape[1]
    K = np.empty((Quu.shape[0], Quu.shape[-1], nx), F32)
    for col in range(nx):
        K[:, :, col] = lu_solve4(LU, piv, -Qxu[:, col, :])
    k = lu_solve4(LU, piv, -qu)
    return K, k


def _value_update(Qxx, Qxu, qx, K, k):
    """V = Q_xx + Q_xu K, v = q_x + Q_xu k (backward_pass_kernel.cu:1027-1041)."""
    V = Qxx.copy()
    v = qx.copy()
    for l in range(K.shape[1]):
        V = V + Qxu[:, :, l, None] * K[:, None, l, :]
        v = v + Qxu[:, :, l] * k[:, l, None]
    return V.astype(F32), v.astype(F32)


def fm_riccati_pnqp(A, B, lxx, luu, lxu, lx, lu, lxxN, lxN, U, u_min, u_max, reg):
    """The forward solve's Riccati pass (backward_pass_kernel.cu:787-1047).
    With bounds (u_min, u_max not None) each step solves the box QP
    min 1/2 du^T Q_uu du + q_u^T du on [u_min - U_t, u_max - U_t] with pnqp4
    from du = 0; its free mask masks Q_uu, Q_xu, q_u, the clamped rows of K
    are zeroed and the clamped entries of k are the PNQP optimum.
    Returns K [B,T,4,nx], k [B,T,4], free mask [B,T,4] (ones without bounds)."""
    Bn, T = A.shape[:2]
    nu = B.shape[-1]
    V = _f(lxxN).copy()
    v = _f(lxN).copy()
    Ks = np.empty((Bn, T, nu, A.shape[-1]), F32)
    ks = np.empty((Bn, T, nu), F32)
    fms = np.ones((Bn, T, nu), F32)
    bounded = u_min is not None and u_max is not None
    for t in range(T - 1, -1, -1):
        Qxx, Qxu, Quu, qx, qu = _q_terms(V, v, A[:, t], B[:, t], lxx[:, t], luu[:, t], lxu[:, t], lx[:, t],
                                         lu[:, t], reg)
        if bounded:
            lo = (_f(u_min)[None, :] - U[:, t]).astype(F32)
            hi = (_f(u_max)[None, :] - U[:, t]).astype(F32)
            dstar, fm = pnqp4(Quu, qu, lo, hi)
            Quu, Qxu, qu = _apply_free_mask(Quu, Qxu, qu, fm)
            K, k = _gains(Quu, Qxu, qu)
            K = (K * fm[:, :, None]).astype(F32)
            k = np.where(fm != 0, k, dstar).astype(F32)
            fms[:, t] = fm
        else:
            K, k = _gains(Quu, Qxu, qu)
        Ks[:, t] = K
        ks[:, t] = k
        V, v = _value_update(Qxx, Qxu, qx, K, k)
    return Ks, ks, fms


def fm_adjoint_riccati(A, B, lxx, luu, lxu, lx, lu, lxxN, lxN, tight, reg):
    """drone_backward_pass_batched on the CUDA path (backward_pass_kernel.cu:
    617-745 via :666-745): Q terms with reg once, then for a tight entry the
    row and column of Q_uu are zeroed with a 1e-11 diagonal, the column of
    Q_xu and the entry of q_u are zeroed; LU gains; V = Q_xx + Q_xu K.
    Returns K, k, v0."""
    Bn, T = A.shape[:2]
    nu = B.shape[-1]
    V = _f(lxxN).copy()
    v = _f(lxN).copy()
    Ks = np.empty((Bn, T, nu, A.shape[-1]), F32)
    ks = np.empty((Bn, T, nu), F32)
    for t in range(T - 1, -1, -1):
        Qxx, Qxu, Quu, qx, qu = _q_terms(V, v, A[:, t], B[:, t], lxx[:, t], luu[:, t], lxu[:, t], lx[:, t],
                                         lu[:, t], reg)
        if tight is not None:
            fm = np.where(np.asarray(tight[:, t], bool), F32(0.0), F32(1.0)).astype(F32)
            Quu, Qxu, qu = _apply_free_mask(Quu, Qxu, qu, fm)
        K, k = _gains(Quu, Qxu, qu)
        Ks[:, t] = K
        ks[:, t] = k
        V, v = _value_update(Qxx, Qxu, qx, K, k)
    return Ks, ks, v


# --------------------------------------------------------------------------
# Line search and solve
# --------------------------------------------------------------------------

def fm_candidates(x0, X, U, K, k, alphas, dt, u_min, u_max, step=None):
    """Candidate rollouts (forward_pass_kernel.cu:123-210): u_t = U_t +
    (alpha k_t + K_t dx_t) with the sum started from alpha k and K's columns
    added in order, clamped, then stepped. Returns Xc [B,nA,T+1,nx], Uc [B,nA,T,nu]."""
    step = fm_step if step is None else step
    Bn, T, nu = U.shape
    nx = X.shape[-1]
    nA = len(alphas)
    Xc = np.empty((Bn, nA, T + 1, nx), F32)
    Uc = np.empty((Bn, nA, T, nu), F32)
    for a, al in enumerate(alphas):
        x = _f(x0).copy()
        Xc[:, a, 0] = x
        for t in range(T):
            dx = (x - X[:, t]).astype(F32)
            du = F32(al) * k[:, t]
            for j in range(nx):
                du = du + K[:, t, :, j] * dx[:, j, None]
            u = (U[:, t] + du).astype(F32)
            if u_min is not None and u_max is not None:
                # fminf(fmaxf(u, lo), hi): a NaN control lands on the lower bound
                u = np.fmin(np.fmax(u, _f(u_min)), _f(u_max)).astype(F32)
            Uc[:, a, t] = u
            x = step(x, u, dt)
            Xc[:, a, t + 1] = x
    return Xc, Uc


def _defaults(B, T, nx, nu, C_f, c_f, x_ref, u_ref):
    n = nx + nu
    C_f = np.zeros((B, n, n), F32) if C_f is None else _f(C_f)
    c_f = np.zeros((B, n), F32) if c_f is None else _f(c_f)
    x_ref = np.zeros((B, T + 1, nx), F32) if x_ref is None else _f(x_ref)
    u_ref = np.zeros((B, T, nu), F32) if u_ref is None else _f(u_ref)
    return C_f, c_f, x_ref, u_ref


def fm_solve(x0, U_init, C, c, C_f=None, c_f=None, x_ref=None, u_ref=None, u_min=None, u_max=None,
             dt=0.05, max_iter=5, reg=1e-6, converge_tol=1e-6, alphas=FM_ALPHAS, forced=None,
             forced_stop=None, step=None, rollout_step=None, jacobian=None):
    """drone_ilqr_solve of the CUDA build (drone_ilqr_ext.cpp:664-1064).

    Returns dict(X, U, tight, X_lin, U_lin, converged, iters_run, trace,
    improvement [iters_run] (the batch maximum per iteration)). X_lin, U_lin
    are the trajectory the last Riccati pass linearised at (the point of the
    returned A_lin, B_lin). `forced` [B, max_iter] replays decisions and
    `forced_stop` the number of iterations the batch ran."""
    step = fm_step if step is None else step
    rollout_step = fm_rollout_step if rollout_step is None else rollout_step
    jacobian = fm_jacobian if jacobian is None else jacobian
    x0 = _f(x0)
    C = _f(C)
    c = _f(c)
    Bn, T, nu = np.shape(U_init)
    nx = x0.shape[-1]
    C_f, c_f, x_ref, u_ref = _defaults(Bn, T, nx, nu, C_f, c_f, x_ref, u_ref)
    bounded = u_min is not None and u_max is not None
    U = _f(U_init).copy()
    if bounded:
        U = np.minimum(np.maximum(U, _f(u_min)), _f(u_max)).astype(F32)
    X = fm_rollout(x0, U, dt, rollout_step)
    best = fm_cost(X, U, C, c, C_f, c_f, x_ref, u_ref, "total")
    trace = np.full((Bn, max_iter), NOT_RUN, np.int64)
    fm = np.ones((Bn, T, nu), F32)
    X_lin, U_lin = X, U
    converged = False
    improvements = []
    it = 0
    for it in range(max_iter):
        X_lin, U_lin = X.copy(), U.copy()
        A, Bm = jacobian(X[:, :T], U, dt)
        lxx, luu, lxu, lx, lu, lxxN, lxN = fm_quadraticize(X, U, C, c, C_f, c_f, x_ref, u_ref)
        K, k, fm = fm_riccati_pnqp(A, Bm, lxx, luu, lxu, lx, lu, lxxN, lxN, U,
                                   u_min if bounded else None, u_max if bounded else None, reg)
        Xc, Uc = fm_candidates(x0, X, U, K, k, alphas, dt, u_min if bounded else None,
                               u_max if bounded else None, step)
        costs = np.stack([fm_cost(Xc[:, a], Uc[:, a], C, c, C_f, c_f, x_ref, u_ref, "line_search")
                          for a in range(len(alphas))], axis=1)
        nan_any = np.isnan(costs).any(axis=1)
        j = np.where(nan_any, np.argmax(np.isnan(costs), axis=1), np.argmin(np.where(np.isnan(costs), np.inf,
                                                                                      costs), axis=1))
        newc = np.where(nan_any, F32(np.nan), costs[np.arange(Bn), j]).astype(F32)
        improved = newc < best
        if forced is not None:
            f = np.asarray(forced[:, it])
            improved = f >= 0
            j = np.where(improved, f, -f - 1)
            newc = np.where(improved, costs[np.arange(Bn), np.clip(j, 0, len(alphas) - 1)], best).astype(F32)
        trace[:, it] = np.where(improved, j, -(j + 1))
        X = np.where(improved[:, None, None], Xc[np.arange(Bn), j], X).astype(F32)
        U = np.where(improved[:, None, None], Uc[np.arange(Bn), j], U).astype(F32)
        new_best = np.where(improved, newc, best).astype(F32)
        imp = np.abs(best - new_best)
        best = new_best
        m = F32(np.nan) if np.isnan(imp).any() else (F32(imp.max()) if Bn else F32(0.0))
        improvements.append(m)
        if it % CHECK_PERIOD == CHECK_PERIOD - 1 or it == max_iter - 1:
            stop = bool(float(m) < converge_tol)
            if forced_stop is not None and it + 1 < max_iter:
                stop = it + 1 == forced_stop
            if stop:
                converged = True
                break
    tight = (fm < F32(0.5)) if bounded else np.zeros((Bn, T, nu), bool)
    return dict(X=X, U=U, tight=tight, X_lin=X_lin, U_lin=U_lin, converged=converged,
                iters_run=it + 1 if max_iter > 0 else 0, trace=trace, improvement=np.array(improvements, F32),
                best_cost=best)


def fm_backward(X, U, X_lin, U_lin, C, grad_X, grad_U, tight, C_f=None, x_ref=None, u_ref=None, dt=0.05,
                reg=1e-6, jacobian=None):
    """DroneMPCFunction.backward of the reference FastMPC
    (differentialMPCPerformance/mpc_compat.py:188-258) on the CUDA path:
    drone_backward_pass_batched (l_x = -dL/dX[:T], l_u = -dL/dU,
    l_xN = -dL/dX_T, l_xxN = C_f[:nx,:nx], A, B at X_lin, U_lin) then
    drone_implicit_diff_assembly (backward_pass_kernel.cu:1092-1256).
    Returns dict(x0, C, c, C_final, c_final, x_ref, u_ref)."""
    jacobian = fm_jacobian if jacobian is None else jacobian
    X = _f(X)
    U = _f(U)
    C = _f(C)
    Bn, T, nu = U.shape
    nx = X.shape[-1]
    n = nx + nu
    C_f, _, x_ref, u_ref = _defaults(Bn, T, nx, nu, C_f, None, x_ref, u_ref)
    A, Bm = jacobian(_f(X_lin)[:, :T], _f(U_lin), dt)
    lxx = C[:, :, :nx, :nx]
    luu = C[:, :, nx:, nx:]
    lxu = C[:, :, :nx, nx:]
    gX = _f(grad_X)
    gU = _f(grad_U)
    K, k, v0 = fm_adjoint_riccati(A, Bm, lxx, luu, lxu, -gX[:, :T], -gU, C_f[:, :nx, :nx], -gX[:, T], tight, reg)
    dX = np.zeros((Bn, T + 1, nx), F32)
    dU = np.zeros((Bn, T, nu), F32)
    for t in range(T):
        du = k[:, t].copy()
        for j in range(nx):
            du = du + K[:, t, :, j] * dX[:, t, j, None]
        dU[:, t] = du
        s = np.zeros((Bn, nx), F32)
        for j in range(nx):
            s = s + A[:, t, :, j] * dX[:, t, j, None]
        for j in range(nu):
            s = s + Bm[:, t, :, j] * du[:, j, None]
        dX[:, t + 1] = s
    tau = np.concatenate([X[:, :T] - x_ref[:, :T], U - u_ref], axis=-1).astype(F32)
    dtau = np.concatenate([dX[:, :T], dU], axis=-1).astype(F32)
    gC = (F32(-0.5) * (dtau[..., :, None] * tau[..., None, :] + tau[..., :, None] * dtau[..., None, :])).astype(F32)
    tauN = np.concatenate([X[:, T] - x_ref[:, T], np.zeros((Bn, nu), F32)], axis=-1).astype(F32)
    dtauN = np.concatenate([dX[:, T], np.zeros((Bn, nu), F32)], axis=-1).astype(F32)
    gCf = (F32(-0.5) * (dtauN[:, :, None] * tauN[:, None, :] + tauN[:, :, None] * dtauN[:, None, :])).astype(F32)
    gxref = np.concatenate([dX[:, :T], dX[:, T:]], axis=1)
    del n
    return dict(x0=(-v0).astype(F32), C=gC, c=(-dtau).astype(F32), C_final=gCf, c_final=(-dtauN).astype(F32),
                x_ref=gxref.astype(F32), u_ref=dU, K=K, k=k, dX=dX)


__all__ = ["FM_ALPHAS", "CHECK_PERIOD", "fm_step", "fm_rollout_step", "fm_jacobian", "fm_rollout", "fm_cost",
           "fm_quadraticize", "lu_factor4", "lu_solve4", "fm_riccati_pnqp", "fm_adjoint_riccati",
           "fm_candidates", "fm_solve", "fm_backward"]
