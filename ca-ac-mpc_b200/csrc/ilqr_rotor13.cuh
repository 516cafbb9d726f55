// ilqr_rotor13.cuh -- the 13-state rotor-thrust quadrotor (device code).
//
// The reference has no such model (its solver and environment use the
// 10-state CTBR DroneDx, acmpc_public-master/diff_mpc_drones/drone.py:409-465);
// DiffMPC's controller takes any f_dyn and linearises it by autodiff
// (DifferentialMPC/controller.py:147-160, 607-615). This is the rigid body of
// the benchmark configurations: state x = [p (3), q = (qw, qx, qy, qz) (4),
// v (3), w (3)], control u = four rotor thrusts as fractions of F_MAX in
// [0, 1], mass 0.75 kg, arm 0.15 m on an X (rotors at (+d,+d), (+d,-d),
// (-d,-d), (-d,+d), d = arm / sqrt 2), inertia diag(2.5e-3, 2.5e-3, 4.5e-3),
// yaw torque KAPPA = 0.016 N m per N of thrust, F_MAX = 8.5 N.
//
//   p' = v
//   q' = 1/2 q (x) (0, w)                       Hamilton product (drone.py:28-33)
//   v' = (F_MAX sum u / m) r(q) - (0, 0, g),    r(q) = q (0,0,1) q*
//   w' = J^-1 (tau(u) - w x J w)
//   x+ = x + dt x'                              explicit Euler, no renormalisation
//
// The step's exact Jacobian is A = I + dt df/dx, B = dt df/du. Every
// expression is written in the same order as the numpy and torch statements
// of the model, and the library is built with -fmad=false, so the step and
// the Jacobian round exactly as those do.
#pragma once

namespace ilqr {
namespace r13 {

constexpr int NX = 13;
constexpr int NU = 4;
constexpr int NT = NX + NU;

// Derived constants, each computed in double precision and rounded once to
// float: F_MAX / m, d F_MAX / Jx, d F_MAX / Jy, KAPPA F_MAX / Jz, the
// gyroscopic ratios (Jy - Jz) / Jx, (Jz - Jx) / Jy, (Jx - Jy) / Jz, and g.
constexpr float FM = 11.333333f;
constexpr float RX = 360.62445f;
constexpr float RY = 360.62445f;
constexpr float RZ = 30.222221f;
constexpr float AX = -0.8f;
constexpr float AY = 0.8f;
constexpr float AZ = 0.0f;
constexpr float GRAV = 9.8066f;

// x' = f(x, u)
__device__ __forceinline__ void xdot(const float* x, const float* u, float* xd) {
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float wx = x[10], wy = x[11], wz = x[12];
  const float u0 = u[0], u1 = u[1], u2 = u[2], u3 = u[3];
  xd[0] = x[7];
  xd[1] = x[8];
  xd[2] = x[9];
  xd[3] = 0.5f * (-qx * wx - qy * wy - qz * wz);
  xd[4] = 0.5f * (qw * wx + qy * wz - qz * wy);
  xd[5] = 0.5f * (qw * wy - qx * wz + qz * wx);
  xd[6] = 0.5f * (qw * wz + qx * wy - qy * wx);
  const float aT = FM * (((u0 + u1) + u2) + u3);
  const float r0 = 2.0f * (qw * qy + qx * qz);
  const float r1 = 2.0f * (qy * qz - qw * qx);
  const float r2 = ((qw * qw - qx * qx) - qy * qy) + qz * qz;
  xd[7] = aT * r0;
  xd[8] = aT * r1;
  xd[9] = aT * r2 - GRAV;
  xd[10] = RX * (((u0 - u1) - u2) + u3) + AX * (wy * wz);
  xd[11] = RY * (((u2 + u3) - u0) - u1) + AY * (wz * wx);
  xd[12] = RZ * (((u0 - u1) + u2) - u3) + AZ * (wx * wy);
}

// x+ = x + dt f(x, u); xn may not alias x.
__device__ __forceinline__ void step(const float* x, const float* u, float dt, float* xn) {
  float xd[NX];
  xdot(x, u, xd);
#pragma unroll
  for (int i = 0; i < NX; ++i) xn[i] = x[i] + dt * xd[i];
}

// Row i of A = I + dt df/dx (a[13]) and of B = dt df/du (b[4]).
__device__ __forceinline__ void jac_row(int i, const float* x, const float* u, float dt, float* a, float* b) {
#pragma unroll
  for (int j = 0; j < NX; ++j) a[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < NU; ++j) b[j] = 0.0f;
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float wx = x[10], wy = x[11], wz = x[12];
  if (i < 3) {  // p' = v
    a[7 + i] = 1.0f * dt;
  } else if (i < 7) {  // q' = 1/2 Omega(w) q = 1/2 Xi(q) w
    const int r = i - 3;
    float om[4], xi[3];
    if (r == 0) {
      om[0] = 0.0f; om[1] = -wx; om[2] = -wy; om[3] = -wz;
      xi[0] = -qx; xi[1] = -qy; xi[2] = -qz;
    } else if (r == 1) {
      om[0] = wx; om[1] = 0.0f; om[2] = wz; om[3] = -wy;
      xi[0] = qw; xi[1] = -qz; xi[2] = qy;
    } else if (r == 2) {
      om[0] = wy; om[1] = -wz; om[2] = 0.0f; om[3] = wx;
      xi[0] = qz; xi[1] = qw; xi[2] = -qx;
    } else {
      om[0] = wz; om[1] = wy; om[2] = -wx; om[3] = 0.0f;
      xi[0] = -qy; xi[1] = qx; xi[2] = qw;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) a[3 + j] = (0.5f * om[j]) * dt;
#pragma unroll
    for (int j = 0; j < 3; ++j) a[10 + j] = (0.5f * xi[j]) * dt;
  } else if (i < 10) {  // v' = aT r(q) - g e3
    const int r = i - 7;
    const float aT = FM * (((u[0] + u[1]) + u[2]) + u[3]);
    float dr[4], rv;
    if (r == 0) {
      dr[0] = qy; dr[1] = qz; dr[2] = qw; dr[3] = qx;
      rv = 2.0f * (qw * qy + qx * qz);
    } else if (r == 1) {
      dr[0] = -qx; dr[1] = -qw; dr[2] = qz; dr[3] = qy;
      rv = 2.0f * (qy * qz - qw * qx);
    } else {
      dr[0] = qw; dr[1] = -qx; dr[2] = -qy; dr[3] = qz;
      rv = ((qw * qw - qx * qx) - qy * qy) + qz * qz;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) a[3 + j] = (aT * (2.0f * dr[j])) * dt;
    const float bv = (FM * rv) * dt;
#pragma unroll
    for (int j = 0; j < NU; ++j) b[j] = bv;
  } else {  // w' = J^-1 (tau - w x J w)
    const int r = i - 10;
    float g;
    int s0, s1, s2, s3;
    if (r == 0) {
      a[11] = (AX * wz) * dt;
      a[12] = (AX * wy) * dt;
      g = RX; s0 = 1; s1 = -1; s2 = -1; s3 = 1;
    } else if (r == 1) {
      a[10] = (AY * wz) * dt;
      a[12] = (AY * wx) * dt;
      g = RY; s0 = -1; s1 = -1; s2 = 1; s3 = 1;
    } else {
      a[10] = (AZ * wy) * dt;
      a[11] = (AZ * wx) * dt;
      g = RZ; s0 = 1; s1 = -1; s2 = 1; s3 = -1;
    }
    b[0] = (s0 > 0 ? g : -g) * dt;
    b[1] = (s1 > 0 ? g : -g) * dt;
    b[2] = (s2 > 0 ? g : -g) * dt;
    b[3] = (s3 > 0 ? g : -g) * dt;
  }
  a[i] = a[i] + 1.0f;
}

}  // namespace r13
}  // namespace ilqr
