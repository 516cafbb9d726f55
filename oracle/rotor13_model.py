"""TEST INFRASTRUCTURE ONLY -- 13-state rotor-thrust quadrotor (numpy).

This model is NOT in the reference: the reference's solver and environment use
the 10-state CTBR model (acmpc_public-master/diff_mpc_drones/drone.py:409-465).
It is the rigid body the benchmark configurations describe (state 13, four
rotor thrusts in [0, 1], mass 0.75 kg, arm 0.15 m, inertia diag
[2.5e-3, 2.5e-3, 4.5e-3]), written here for DiffMPC's model-generic path
(DifferentialMPC/controller.py:147-160, 607-615 with GradMethod.AUTO_DIFF).
The solver arithmetic around it is the DiffMPC restatement in
diffmpc_oracle.py; parity of that solver on this model is pinned by golden
vectors from DiffMPC itself (tests/golden/make_rotor13_golden.py), while the
model itself is pinned by nothing in the reference ("model unpinned by the
reference").

State x = [p (3), q = (qw, qx, qy, qz) (4), v (3), w (3)] in the world frame
for p, v and the body frame for w; control u = four rotor thrusts as fractions
of F_MAX. Rotors sit on an X at (+d, +d), (+d, -d), (-d, -d), (-d, +d) with
d = arm / sqrt(2); rotors 0 and 2 spin one way, 1 and 3 the other, with yaw
torque KAPPA per newton of thrust. Continuous dynamics:

    p' = v
    q' = 1/2 q (x) (0, w)                      (Hamilton product, drone.py:28-33 order)
    v' = (F_MAX sum(u) / m) r(q) + (0, 0, -g)  r(q) = q (0,0,1) q* (drone.py:145-156)
    w' = J^-1 (tau(u) - w x J w)

    r(q) = [2 (qw qy + qx qz), 2 (qy qz - qw qx), qw^2 - qx^2 - qy^2 + qz^2]
    tau  = F_MAX [d (u0 - u1 - u2 + u3), d (-u0 - u1 + u2 + u3), KAPPA (u0 - u1 + u2 - u3)]

Discrete step: explicit Euler, x+ = x + dt x' (no quaternion renormalisation),
so its Jacobian is exactly A = I + dt df/dx, B = dt df/du.
"""

from __future__ import annotations

import numpy as np

from .diffmpc_oracle import Model

NX13, NU13 = 13, 4
MASS13 = 0.75
ARM13 = 0.15
INERTIA13 = (2.5e-3, 2.5e-3, 4.5e-3)
KAPPA13 = 0.016
F_MAX13 = 8.5
GRAV13 = 9.8066
HOVER_U13 = MASS13 * GRAV13 / (4.0 * F_MAX13)


def rotor13_constants(dtype=np.float32):
    """The model's derived constants, each computed in float64 and rounded
    once to ``dtype`` (the CUDA kernels hold the same float32 values):
    FM = F_MAX / m, RX = d F_MAX / Jx, RY = d F_MAX / Jy, RZ = KAPPA F_MAX / Jz,
    AX = (Jy - Jz) / Jx, AY = (Jz - Jx) / Jy, AZ = (Jx - Jy) / Jz, G."""
    jx, jy, jz = INERTIA13
    d = ARM13 / np.sqrt(2.0)
    vals = dict(FM=F_MAX13 / MASS13, RX=d * F_MAX13 / jx, RY=d * F_MAX13 / jy,
                RZ=KAPPA13 * F_MAX13 / jz, AX=(jy - jz) / jx, AY=(jz - jx) / jy,
                AZ=(jx - jy) / jz, G=GRAV13)
    return {k: np.dtype(dtype).type(v) for k, v in vals.items()}


def rotor13_xdot(x, u):
    """Continuous dynamics f(x, u) for x [B,13], u [B,4] -> [B,13]."""
    dtype = x.dtype
    k = rotor13_constants(dtype)
    half = dtype.type(0.5)
    two = dtype.type(2.0)
    qw, qx, qy, qz = x[:, 3], x[:, 4], x[:, 5], x[:, 6]
    v = x[:, 7:10]
    wx, wy, wz = x[:, 10], x[:, 11], x[:, 12]
    u0, u1, u2, u3 = u[:, 0], u[:, 1], u[:, 2], u[:, 3]
    qd = np.stack([half * (-qx * wx - qy * wy - qz * wz),
                   half * (qw * wx + qy * wz - qz * wy),
                   half * (qw * wy - qx * wz + qz * wx),
                   half * (qw * wz + qx * wy - qy * wx)], axis=1)
    aT = k["FM"] * (((u0 + u1) + u2) + u3)
    r0 = two * (qw * qy + qx * qz)
    r1 = two * (qy * qz - qw * qx)
    r2 = ((qw * qw - qx * qx) - qy * qy) + qz * qz
    vd = np.stack([aT * r0, aT * r1, aT * r2 - k["G"]], axis=1)
    wd = np.stack([k["RX"] * (((u0 - u1) - u2) + u3) + k["AX"] * (wy * wz),
                   k["RY"] * (((u2 + u3) - u0) - u1) + k["AY"] * (wz * wx),
                   k["RZ"] * (((u0 - u1) + u2) - u3) + k["AZ"] * (wx * wy)], axis=1)
    return np.concatenate([v, qd, vd, wd], axis=1)


def rotor13_step(x, u, dt):
    """x+ = x + dt f(x, u) for x [B,13], u [B,4]."""
    dtype = x.dtype
    return x + dtype.type(dt) * rotor13_xdot(x, u)


def rotor13_jacobian(x, u, dt):
    """A = I + dt df/dx [B,13,13], B = dt df/du [B,13,4] of rotor13_step."""
    dtype = x.dtype
    k = rotor13_constants(dtype)
    nb = x.shape[0]
    half = dtype.type(0.5)
    two = dtype.type(2.0)
    Jx = np.zeros((nb, NX13, NX13), dtype=dtype)
    Ju = np.zeros((nb, NX13, NU13), dtype=dtype)
    qw, qx, qy, qz = x[:, 3], x[:, 4], x[:, 5], x[:, 6]
    wx, wy, wz = x[:, 10], x[:, 11], x[:, 12]
    z = np.zeros_like(qw)
    for i in range(3):                      # p' = v
        Jx[:, i, 7 + i] = 1.0
    Om = [[z, -wx, -wy, -wz], [wx, z, wz, -wy], [wy, -wz, z, wx], [wz, wy, -wx, z]]
    Xi = [[-qx, -qy, -qz], [qw, -qz, qy], [qz, qw, -qx], [-qy, qx, qw]]
    for i in range(4):                      # q' = 1/2 Omega(w) q = 1/2 Xi(q) w
        for j in range(4):
            Jx[:, 3 + i, 3 + j] = half * Om[i][j]
        for j in range(3):
            Jx[:, 3 + i, 10 + j] = half * Xi[i][j]
    aT = k["FM"] * (((u[:, 0] + u[:, 1]) + u[:, 2]) + u[:, 3])
    dr = [[qy, qz, qw, qx], [-qx, -qw, qz, qy], [qw, -qx, -qy, qz]]
    r = [two * (qw * qy + qx * qz), two * (qy * qz - qw * qx),
         ((qw * qw - qx * qx) - qy * qy) + qz * qz]
    for i in range(3):                      # v' = aT r(q) - g e3
        for j in range(4):
            Jx[:, 7 + i, 3 + j] = aT * (two * dr[i][j])
            Ju[:, 7 + i, j] = k["FM"] * r[i]
    Jx[:, 10, 11] = k["AX"] * wz            # w' gyroscopic term
    Jx[:, 10, 12] = k["AX"] * wy
    Jx[:, 11, 10] = k["AY"] * wz
    Jx[:, 11, 12] = k["AY"] * wx
    Jx[:, 12, 10] = k["AZ"] * wy
    Jx[:, 12, 11] = k["AZ"] * wx
    mix = [(k["RX"], (1, -1, -1, 1)), (k["RY"], (-1, -1, 1, 1)), (k["RZ"], (1, -1, 1, -1))]
    for i, (g, sg) in enumerate(mix):
        for j in range(4):
            Ju[:, 10 + i, j] = g if sg[j] > 0 else -g
    dtt = dtype.type(dt)
    A = Jx * dtt + np.eye(NX13, dtype=dtype)[None]
    Bm = Ju * dtt
    return A, Bm


ROTOR13 = Model("rotor13", NX13, NU13, rotor13_step, rotor13_jacobian)

__all__ = ["NX13", "NU13", "MASS13", "ARM13", "INERTIA13", "KAPPA13", "F_MAX13", "GRAV13",
           "HOVER_U13", "rotor13_constants", "rotor13_xdot", "rotor13_step", "rotor13_jacobian",
           "ROTOR13"]
