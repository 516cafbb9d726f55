// ilqr_fastmpc.cu -- the FastMPC numerics mode: the solver as the reference
// FastMPC extension's CUDA build runs it (differentialMPCPerformance/cpp/
// drone_ilqr_ext.cpp:664-1064 solve loop; backward_pass_kernel.cu:787-1047
// PNQP-aware Riccati pass; forward_pass_kernel.cu:66-210 line search and
// model step; drone_kernels.cu:64-250 Jacobian and initial rollout;
// backward_pass_kernel.cu:617-745 masked adjoint Riccati and :1092-1256
// implicit-diff assembly), for the 10-state CTBR quadrotor.
//
// Layout: one batch element per group of 16 lanes, two elements per warp,
// four warps per CTA. Riccati step (lane i < 10 owns row i of V, Q_xx, Q_xu;
// lanes 10..13 own the control rows of Q_uu, q_u):
//   J   A_t, B_t entries from the linearisation point (a 36-entry table, three
//       per lane, plus the thrust column), cost rows from C
//   P1  (V A)_i., (V B)_i.
//   P2  Q_xx,i. = C_xx,i. + A_.i^T (V A); Q_xu,i.; q_x,i; q_u,j on lane
//       10 + j; Q_uu entry (l / 4, l % 4) on lane l of all 16
//   P3  every lane solves the step's box QP with PNQP-4 (same inputs, same
//       answer), masks Q_uu, Q_xu, q_u with its free mask, factors Q_uu by
//       the reference's pivoted LU and solves its column of K; k likewise
//   P4  V_i. = Q_xx,i. + Q_xu,i. K ; v_i = q_x,i + Q_xu,i. k
// with a group barrier after each. The line search runs candidate a on lane
// a (alpha_a), into its own workspace slot; accepting re-points the nominal.
//
// The batch stops as one (drone_ilqr_ext.cpp:1029-1049): the iterations run
// in segments of four, one launch each; after a segment a one-CTA kernel
// reduces the elements' last improvements and sets the stop flag that the
// next segment reads. An element that fails to improve recomputes the same
// candidates on every later iteration, so it is frozen at its first
// rejection (its trace repeats that rejection).
//
// Arithmetic is fp32. The matrix-product and cost sums run in index order as
// fused multiply-adds, and this file is compiled with -prec-div=false, so
// divisions (PNQP, the LU, the model step) are the approximate 2-ulp kind: the
// reference build compiles with --use_fast_math, which does both. The oracle
// rounds each product and divides exactly, so the two differ at the rounding
// level. The model step and Jacobian entries are otherwise evaluated without
// contraction (the library is compiled with -fmad=false).
#include <cstdint>

#include "ilqr_b200.h"
#include "ilqr_device.cuh"
#include "ilqr_kernels.h"
#include "ilqr_pnqp.cuh"

namespace ilqr {
namespace fm {

namespace {

constexpr int NXf = 10;
constexpr int NUf = 4;
constexpr int Nf = 14;
constexpr int NN = Nf * Nf;
constexpr int GL = 16;             // lanes per element
constexpr int EPW = 2;             // elements per warp
constexpr int WPC = 4;             // warps per CTA
constexpr int EPC = EPW * WPC;     // elements per CTA
constexpr int THREADS = WPC * 32;
constexpr int REC = 16;            // floats per trajectory record: x[10], u[4], 2 pad
constexpr int KREC = 44;           // floats per gain record: K[4][10], k[4]
constexpr unsigned SM_COUNT_FM = 148;  // B200 SMs (the register-tier choice)
constexpr float MASS = 0.752f;     // drone_kernels.cu:12
constexpr float G_VAL = -9.8066f;  // drone_kernels.cu:13

// Per-element shared memory (floats).
constexpr int S_A = 0;       // A_t [10][10]
constexpr int S_B = 100;     // B_t [10][4]
constexpr int S_VA = 140;    // V A [10][10]
constexpr int S_VB = 240;    // V B [10][4]
constexpr int S_V = 280;     // v [10]
constexpr int S_QUU = 290;   // Q_uu [4][4]
constexpr int S_QU = 306;    // q_u [4]
constexpr int S_K = 310;     // K_t [4][10]
constexpr int S_Z = 350;     // linearisation point x_t, u_t [14]
constexpr int S_EZ = 364;    // x_t - x_ref_t, u_t - u_ref_t [14]
constexpr int S_JV = 378;    // Jacobian variables [11]
constexpr int S_DX = 390;    // backward sweep: dX_t [10]
constexpr int S_DU = 400;    // dU_t [4]
constexpr int S_ELEM = 432;  // 432 = 16 mod 32: the warp's two elements use opposite bank halves

// Jacobian table: entry e -> value written to the element block.
//   bits 0..8 destination offset, 9..12 variable, 13 coefficient (0: dt/2,
//   1: 2 dt), 14 form (0: 0 +- p, 1: +-p), 15 sign (1: minus).
// Variables: 0..2 w, 3..6 q, 7..10 q * fc / m. Entries follow
// drone_kernels.cu:124-183.
constexpr uint32_t jt(int dest, int var, int coef, int form, int minus) {
  return (uint32_t)dest | ((uint32_t)var << 9) | ((uint32_t)coef << 13) | ((uint32_t)form << 14) |
         ((uint32_t)minus << 15);
}
#define A_(r, c) (S_A + (r) * 10 + (c))
#define B_(r, c) (S_B + (r) * 4 + (c))
__device__ const uint32_t kJacTable[36] = {
    // quaternion block of A: 0 -+ dt/2 * w
    jt(A_(3, 4), 0, 0, 0, 1), jt(A_(3, 5), 1, 0, 0, 1), jt(A_(3, 6), 2, 0, 0, 1),
    jt(A_(4, 3), 0, 0, 0, 0), jt(A_(4, 5), 2, 0, 0, 0), jt(A_(4, 6), 1, 0, 0, 1),
    jt(A_(5, 3), 1, 0, 0, 0), jt(A_(5, 4), 2, 0, 0, 1), jt(A_(5, 6), 0, 0, 0, 0),
    jt(A_(6, 3), 2, 0, 0, 0), jt(A_(6, 4), 1, 0, 0, 0), jt(A_(6, 5), 0, 0, 0, 1),
    // quaternion rows of B: +-dt/2 * q
    jt(B_(3, 1), 4, 0, 1, 1), jt(B_(3, 2), 5, 0, 1, 1), jt(B_(3, 3), 6, 0, 1, 1),
    jt(B_(4, 1), 3, 0, 1, 0), jt(B_(4, 2), 6, 0, 1, 1), jt(B_(4, 3), 5, 0, 1, 0),
    jt(B_(5, 1), 6, 0, 1, 0), jt(B_(5, 2), 3, 0, 1, 0), jt(B_(5, 3), 4, 0, 1, 1),
    jt(B_(6, 1), 5, 0, 1, 1), jt(B_(6, 2), 4, 0, 1, 0), jt(B_(6, 3), 3, 0, 1, 0),
    // velocity rows of A: +-2 dt * q_k fc / m
    jt(A_(7, 3), 9, 1, 1, 0), jt(A_(7, 4), 10, 1, 1, 0), jt(A_(7, 5), 7, 1, 1, 0), jt(A_(7, 6), 8, 1, 1, 0),
    jt(A_(8, 3), 8, 1, 1, 1), jt(A_(8, 4), 7, 1, 1, 1), jt(A_(8, 5), 10, 1, 1, 0), jt(A_(8, 6), 9, 1, 1, 0),
    jt(A_(9, 3), 7, 1, 1, 0), jt(A_(9, 4), 8, 1, 1, 1), jt(A_(9, 5), 9, 1, 1, 1), jt(A_(9, 6), 10, 1, 1, 0),
};
#undef A_
#undef B_

__device__ __forceinline__ float fclamp(float u, float lo, float hi) { return fminf(fmaxf(u, lo), hi); }

// Initial clamp of U_init (at::clamp, drone_ilqr_ext.cpp:714-716): NaN stays NaN.
__device__ __forceinline__ float nan_clamp(float u, float lo, float hi) {
  return u != u ? u : fminf(fmaxf(u, lo), hi);
}

// ---- the extension's model step -------------------------------------------

__device__ __forceinline__ void quat_step(const float* x, float wx, float wy, float wz, float dt, float* xo) {
  // exp_map (forward_pass_kernel.cu:26-39), product and renormalisation (:86-99)
  const float w_norm = sqrtf(wx * wx + wy * wy + wz * wz) + 1e-8f;
  const float half = w_norm * (dt * 0.5f);
  const float s = sinf(half);
  const float c = cosf(half);
  const float inv = 1.0f / w_norm;
  const float ew = c, ex = wx * inv * s, ey = wy * inv * s, ez = wz * inv * s;
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float nw = qw * ew - qx * ex - qy * ey - qz * ez;
  const float nx = qw * ex + qx * ew + qy * ez - qz * ey;
  const float ny = qw * ey - qx * ez + qy * ew + qz * ex;
  const float nz = qw * ez + qx * ey - qy * ex + qz * ew;
  const float qn = sqrtf(nw * nw + nx * nx + ny * ny + nz * nz) + 1e-8f;
  xo[3] = nw / qn;
  xo[4] = nx / qn;
  xo[5] = ny / qn;
  xo[6] = nz / qn;
}

// Line-search step (forward_pass_kernel.cu:66-115): cross-product rotation of
// the body thrust by the old quaternion. x and xo may alias.
__device__ __forceinline__ void step_cross(const float* x, const float* u, float dt, float* xo) {
  float y[10];
  const float fc = u[0];
  y[0] = x[0] + x[7] * dt;
  y[1] = x[1] + x[8] * dt;
  y[2] = x[2] + x[9] * dt;
  quat_step(x, u[1], u[2], u[3], dt, y);
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float zero = 0.0f;
  const float tx = qy * fc - qz * zero;
  const float ty = qz * zero - qx * fc;
  const float tz = qx * zero - qy * zero;
  const float ttx = qy * tz - qz * ty;
  const float tty = qz * tx - qx * tz;
  const float ttz = qx * ty - qy * tx;
  const float ax = (zero + 2.0f * (qw * tx + ttx)) / MASS;
  const float ay = (zero + 2.0f * (qw * ty + tty)) / MASS;
  const float az = (fc + 2.0f * (qw * tz + ttz)) / MASS + G_VAL;
  y[7] = x[7] + ax * dt;
  y[8] = x[8] + ay * dt;
  y[9] = x[9] + az * dt;
#pragma unroll
  for (int i = 0; i < 10; ++i) xo[i] = y[i];
}

// Initial-rollout step (drone_kernels.cu:195-250): rotation-matrix form.
__device__ __forceinline__ void step_matrix(const float* x, const float* u, float dt, float* xo) {
  float y[10];
  const float fc = u[0];
  y[0] = x[0] + x[7] * dt;
  y[1] = x[1] + x[8] * dt;
  y[2] = x[2] + x[9] * dt;
  quat_step(x, u[1], u[2], u[3], dt, y);
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float zero = 0.0f, two = 2.0f;
  const float q00 = qw * qw, q11 = qx * qx, q22 = qy * qy, q33 = qz * qz;
  const float q01 = qw * qx, q02 = qw * qy, q03 = qw * qz;
  const float q12 = qx * qy, q13 = qx * qz, q23 = qy * qz;
  const float rx = (q00 + q11 - q22 - q33) * zero + two * (q12 - q03) * zero + two * (q13 + q02) * fc;
  const float ry = two * (q12 + q03) * zero + (q00 - q11 + q22 - q33) * zero + two * (q23 - q01) * fc;
  const float rz = two * (q13 - q02) * zero + two * (q23 + q01) * zero + (q00 - q11 - q22 + q33) * fc;
  y[7] = x[7] + (rx / MASS) * dt;
  y[8] = x[8] + (ry / MASS) * dt;
  y[9] = x[9] + (rz / MASS + G_VAL) * dt;
#pragma unroll
  for (int i = 0; i < 10; ++i) xo[i] = y[i];
}

// ---- the extension's 4 x 4 LU (backward_pass_kernel.cu:420-470) ------------

__device__ __forceinline__ void lu_factor4(float (&A)[4][4], int (&piv)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int mr = k;
    float mv = fabsf(A[k][k]);
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      const float v = fabsf(A[i][k]);
      if (v > mv) {
        mv = v;
        mr = i;
      }
    }
    piv[k] = mr;
    // row swap with compile-time indices (mr is runtime)
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      if (i == mr) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float t = A[k][j];
          A[k][j] = A[i][j];
          A[i][j] = t;
        }
      }
    }
    float pv = A[k][k];
    if (fabsf(pv) < 1e-10f) pv = pv < 0.0f ? -1e-10f : 1e-10f;
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      A[i][k] = A[i][k] / pv;
#pragma unroll
      for (int j = k + 1; j < 4; ++j) A[i][j] = A[i][j] - A[i][k] * A[k][j];
    }
  }
}

__device__ __forceinline__ void lu_solve4(const float (&LU)[4][4], const int (&piv)[4], float (&b)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      if (piv[k] == i) {
        const float t = b[k];
        b[k] = b[i];
        b[i] = t;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int i = k + 1; i < 4; ++i) b[i] = b[i] - LU[i][k] * b[k];
  }
#pragma unroll
  for (int i = 3; i >= 0; --i) {
    float s = b[i];
#pragma unroll
    for (int j = i + 1; j < 4; ++j) s = s - LU[i][j] * b[j];
    b[i] = s / LU[i][i];
  }
}

__device__ __forceinline__ float pick4(const float (&a)[4], int i) {
  float r = a[0];
#pragma unroll
  for (int q = 1; q < 4; ++q) r = (q == i) ? a[q] : r;
  return r;
}

__device__ __forceinline__ float pick_alpha(const float (&al)[ILQR_MAX_ALPHAS_DEV], int i) {
  float r = al[0];
#pragma unroll
  for (int q = 1; q < ILQR_MAX_ALPHAS_DEV; ++q) r = (q == i) ? al[q] : r;
  return r;
}

struct Group {
  float* sm;
  unsigned gm;  // the group's lanes
  int l;        // lane within the group
  int base;     // first warp lane of the group
  __device__ __forceinline__ void sync() const { __syncwarp(gm); }
};

// Writes the initial A (identity, dt at (0,7), (1,8), (2,9)) and B (zero);
// the Jacobian table overwrites its entries each step, the rest never changes.
__device__ __forceinline__ void init_jacobian(const Group& G, float dt) {
  for (int e = G.l; e < 140; e += GL) {
    float v = 0.0f;
    if (e < 100) {
      const int r = e / 10, c = e % 10;
      if (r == c) v = 1.0f;
      if ((r == 0 && c == 7) || (r == 1 && c == 8) || (r == 2 && c == 9)) v = dt;
    }
    G.sm[S_A + e] = v;
  }
}

// J phase: A_t, B_t at the point in S_Z (drone_kernels.cu:124-190).
__device__ __forceinline__ void jacobian(const Group& G, const uint32_t* jtab, float dt) {
  float* sm = G.sm;
  const int l = G.l;
  const float fc = sm[S_Z + 10];
  if (l < 3) {
    sm[S_JV + l] = sm[S_Z + 11 + l];
  } else if (l < 7) {
    sm[S_JV + l] = sm[S_Z + l];
  } else if (l < 11) {
    const float fcm = fc / MASS;
    sm[S_JV + l] = sm[S_Z + l - 4] * fcm;
  }
  G.sync();
  const float h = 0.5f * dt;
  const float t2 = 2.0f * dt;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int e = l + GL * r;
    if (e < 36) {
      const uint32_t code = jtab[e];
      const float var = sm[S_JV + ((code >> 9) & 15u)];
      const float p = (((code >> 13) & 1u) ? t2 : h) * var;
      const bool minus = (code >> 15) & 1u;
      float v;
      if (((code >> 14) & 1u) == 0u) {
        v = minus ? 0.0f - p : 0.0f + p;
      } else {
        v = minus ? -p : p;
      }
      sm[code & 511u] = v;
    }
  }
  if (l >= 13) {
    const float qw = sm[S_Z + 3], qx = sm[S_Z + 4], qy = sm[S_Z + 5], qz = sm[S_Z + 6];
    const float dtm = dt / MASS;
    float v;
    if (l == 13) {
      v = 2.0f * (qx * qz + qw * qy) * dtm;
    } else if (l == 14) {
      v = 2.0f * (qy * qz - qw * qx) * dtm;
    } else {
      v = (qw * qw - qx * qx - qy * qy + qz * qz) * dtm;
    }
    sm[S_B + (l - 6) * 4] = v;
  }
  G.sync();
}

// Loads the record rec (x[10], u[4]) into S_Z and z - ref into S_EZ; the
// terminal record (u absent) when terminal.
__device__ __forceinline__ void load_point(const Group& G, const float* rec, const float* xr, const float* ur,
                                          bool terminal) {
  const int l = G.l;
  if (l < Nf) {
    float z = 0.0f, e = 0.0f;
    if (l < NXf) {
      z = rec[l];
      e = z - (xr != nullptr ? xr[l] : 0.0f);
    } else if (!terminal) {
      z = rec[l];
      e = z - (ur != nullptr ? ur[l - NXf] : 0.0f);
    }
    G.sm[S_Z + l] = z;
    G.sm[S_EZ + l] = e;
  }
  G.sync();
}

// C_uu entry (l / 4, l % 4) of a step's 14x14 cost block, for group lane l.
__device__ __forceinline__ float quu_entry(const float* __restrict__ cs, int l) {
  return __ldg(cs + (NXf + (l >> 2)) * Nf + NXf + (l & 3));
}

// One Riccati step (P1..P4) on the A_t, B_t and Q inputs already set up.
//   lane i < 10: Vr = V row i, cx = C row i (l_xx row, l_xu row), lxi = l_x,i
//   lane 10 + j: luj = l_u,j
//   every lane l: cq = C_uu entry (l / 4, l % 4) (quu_entry)
// MODE 0: unmasked; 1: PNQP free mask (forward solve); 2: tight mask
// (adjoint). Outputs K_t, k_t into the gain record and (MODE 1) the free mask.
template <int MODE>
__device__ __forceinline__ void riccati_step(const Group& G, float (&Vr)[NXf], const float (&cx)[Nf], float lxi,
                                            float cq, float luj, float reg, const float* umin,
                                            const float* umax, const uint8_t* tight_row, float* krec,
                                            float* fm_row) {
  float* sm = G.sm;
  const int l = G.l;
  const bool xrow = l < NXf;
  const bool urow = l >= NXf && l < Nf;
  // The matrix products run two columns per packed FP32 instruction (the
  // same sums in the same order; rows of A, B, V A, V B and K start on even
  // offsets, so a column pair is one 8-byte shared load).
  // P1: (V A)_i., (V B)_i.
  if (xrow) {
    float2 v2[NXf];
#pragma unroll
    for (int k = 0; k < NXf; ++k) v2[k] = dup2(Vr[k]);
#pragma unroll
    for (int j = 0; j < NXf; j += 2) {
      float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < NXf; ++k) s = fma2(v2[k], ld2(sm + S_A + k * 10 + j), s);
      *reinterpret_cast<float2*>(sm + S_VA + l * 10 + j) = s;
    }
#pragma unroll
    for (int j = 0; j < NUf; j += 2) {
      float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < NXf; ++k) s = fma2(v2[k], ld2(sm + S_B + k * 4 + j), s);
      *reinterpret_cast<float2*>(sm + S_VB + l * 4 + j) = s;
    }
  }
  G.sync();
  // P2
  float Qxx[NXf] = {}, Qxu[NUf] = {}, qx = 0.0f;
  if (xrow) {
    float2 a2[NXf];  // column l of A
#pragma unroll
    for (int k = 0; k < NXf; ++k) a2[k] = dup2(sm[S_A + k * 10 + l]);
#pragma unroll
    for (int j = 0; j < NXf; j += 2) {
      float2 s = make_float2(cx[j], cx[j + 1]);
#pragma unroll
      for (int k = 0; k < NXf; ++k) s = fma2(a2[k], ld2(sm + S_VA + k * 10 + j), s);
      Qxx[j] = s.x;
      Qxx[j + 1] = s.y;
    }
#pragma unroll
    for (int j = 0; j < NUf; j += 2) {
      float2 s = make_float2(cx[NXf + j], cx[NXf + j + 1]);
#pragma unroll
      for (int k = 0; k < NXf; ++k) s = fma2(a2[k], ld2(sm + S_VB + k * 4 + j), s);
      Qxu[j] = s.x;
      Qxu[j + 1] = s.y;
    }
    float s = lxi;
#pragma unroll
    for (int k = 0; k < NXf; ++k) s = fmaf(sm[S_A + k * 10 + l], sm[S_V + k], s);
    qx = s;
  } else if (urow) {
    const int j = l - NXf;
    float s = luj;
#pragma unroll
    for (int k = 0; k < NXf; ++k) s = fmaf(sm[S_B + k * 4 + j], sm[S_V + k], s);
    sm[S_QU + j] = s;
  }
  {  // Q_uu entry (j, m) = (l / 4, l % 4) on every lane: 16 entries, 16 lanes
    const int j = l >> 2, m = l & 3;
    float s = cq;
#pragma unroll
    for (int k = 0; k < NXf; ++k) s = fmaf(sm[S_B + k * 4 + j], sm[S_VB + k * 4 + m], s);
    if (m == j) s = s + reg;
    sm[S_QUU + l] = s;
  }
  G.sync();
  // P3: mask, factor, gains
  float H[4][4], q[4], fr[4] = {1.0f, 1.0f, 1.0f, 1.0f}, dstar[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) H[i][j] = sm[S_QUU + i * 4 + j];
    q[i] = sm[S_QU + i];
  }
  if (MODE == 1) {
    float lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float ut = sm[S_Z + NXf + i];
      lo[i] = __ldg(umin + i) - ut;
      hi[i] = __ldg(umax + i) - ut;
    }
    pnqp::pnqp4(H, q, lo, hi, dstar, fr);
  } else if (MODE == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) fr[i] = tight_row[i] ? 0.0f : 1.0f;
  }
  if (MODE != 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) H[i][j] = H[i][j] * (fr[i] * fr[j]);
      if (fr[i] == 0.0f) H[i][i] = H[i][i] + 1e-11f;
      q[i] = q[i] * fr[i];
    }
#pragma unroll
    for (int j = 0; j < NUf; ++j) Qxu[j] = Qxu[j] * fr[j];
  }
  int piv[4];
  lu_factor4(H, piv);
  if (xrow) {
    float rhs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rhs[i] = -Qxu[i];
    lu_solve4(H, piv, rhs);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float kv = MODE == 1 ? rhs[i] * fr[i] : rhs[i];
      sm[S_K + i * 10 + l] = kv;
      krec[i * 10 + l] = kv;
    }
  }
  float kk[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) kk[i] = -q[i];
  lu_solve4(H, piv, kk);
  if (MODE == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) kk[i] = fr[i] != 0.0f ? kk[i] : dstar[i];
  }
  if (urow) {
    const int j = l - NXf;
    krec[40 + j] = pick4(kk, j);
    if (fm_row != nullptr) fm_row[j] = pick4(fr, j);
  }
  G.sync();
  // P4: V = Q_xx + Q_xu K, v = q_x + Q_xu k (the masked Q_xu)
  if (xrow) {
    float2 u2[NUf];
#pragma unroll
    for (int m = 0; m < NUf; ++m) u2[m] = dup2(Qxu[m]);
#pragma unroll
    for (int j = 0; j < NXf; j += 2) {
      float2 s = make_float2(Qxx[j], Qxx[j + 1]);
#pragma unroll
      for (int m = 0; m < NUf; ++m) s = fma2(u2[m], ld2(sm + S_K + m * 10 + j), s);
      Vr[j] = s.x;
      Vr[j + 1] = s.y;
    }
    float s = qx;
#pragma unroll
    for (int m = 0; m < NUf; ++m) s = fmaf(Qxu[m], kk[m], s);
    sm[S_V + l] = s;
  }
  G.sync();
}

// Cost rows of step t for the Riccati lanes: C row i (lane i < 10) or C_uu
// row j (lane 10 + j), and l_x,i / l_u,j from the errors in S_EZ
// (drone_ilqr_ext.cpp:808-816). cs: C of the step, cv: c of the step.
__device__ __forceinline__ void cost_rows(const Group& G, const float* __restrict__ cs,
                                          const float* __restrict__ cv, float (&cx)[Nf], float& lxi,
                                          float (&cu)[NUf], float& luj) {
  const float* sm = G.sm;
  const int l = G.l;
  if (l < NXf) {
#pragma unroll
    for (int j = 0; j < Nf; ++j) cx[j] = __ldg(cs + l * Nf + j);
    float a = cx[0] * sm[S_EZ + 0];
#pragma unroll
    for (int j = 1; j < NXf; ++j) a = fmaf(cx[j], sm[S_EZ + j], a);
    float b = cx[NXf] * sm[S_EZ + NXf];
#pragma unroll
    for (int j = 1; j < NUf; ++j) b = fmaf(cx[NXf + j], sm[S_EZ + NXf + j], b);
    lxi = a + b + __ldg(cv + l);
  } else if (l < Nf) {
    const int j = l - NXf;
#pragma unroll
    for (int m = 0; m < NUf; ++m) cu[m] = __ldg(cs + l * Nf + NXf + m);
    float a = __ldg(cs + NXf + j) * sm[S_EZ + 0];
#pragma unroll
    for (int k = 1; k < NXf; ++k) a = fmaf(__ldg(cs + k * Nf + NXf + j), sm[S_EZ + k], a);
    float b = cu[0] * sm[S_EZ + NXf];
#pragma unroll
    for (int m = 1; m < NUf; ++m) b = fmaf(cu[m], sm[S_EZ + NXf + m], b);
    luj = a + b + __ldg(cv + l);
  }
}

// 0.5 z^T C z and z^T c, each summed in index order, with the rows of C z
// split over L lanes: this lane (r of the L lanes starting at warp lane
// `first`) forms rows r, r + L, ...; the 14 row terms are gathered by shuffles,
// so every one of the L lanes returns the same sums. form 0: 0.5 * sum(z Cz)
// (compute_cost), form 1: sum(0.5 * (z Cz)) (line search). A null C or c
// reads as zeros (the zero terminal cost of the operator).
template <int L>
__device__ __forceinline__ void quad_split(const float* __restrict__ Cm, const float* __restrict__ cv,
                                           const float (&z)[Nf], int r, unsigned gm, int first, int form,
                                           float& quad, float& lin) {
  constexpr int RPL = (Nf + L - 1) / L;
  float tr[RPL];
#pragma unroll
  for (int k = 0; k < RPL; ++k) {
    const int i = r + k * L;
    float term = 0.0f;
    if (i < Nf) {
      const float* row = Cm + i * Nf;
      auto ld = [&](int j) { return Cm != nullptr ? __ldg(row + j) : 0.0f; };
      float cz = ld(0) * z[0];
#pragma unroll
      for (int j = 1; j < Nf; ++j) cz = fmaf(ld(j), z[j], cz);
      float zi = z[0];
#pragma unroll
      for (int q = 1; q < Nf; ++q) zi = (q == i) ? z[q] : zi;
      term = form == 0 ? zi * cz : 0.5f * (zi * cz);
    }
    tr[k] = term;
  }
  float sq = 0.0f, sl = 0.0f;
#pragma unroll
  for (int i = 0; i < Nf; ++i) {
    const float v = __shfl_sync(gm, tr[i / L], first + i % L);
    sq = i == 0 ? v : sq + v;
    const float lt = z[i] * (cv != nullptr ? __ldg(cv + i) : 0.0f);
    sl = i == 0 ? lt : sl + lt;
  }
  quad = form == 0 ? 0.5f * sq : sq;
  lin = sl;
}

}  // namespace

// ---------------------------------------------------------------------------
// Solve
// ---------------------------------------------------------------------------

// LPC lanes per line-search candidate (4 for up to four step sizes, else 2).
// MINB CTAs per SM: the register tier (2: up to 255 registers, for grids of one
// 2-CTA wave; 3: 168 registers, for larger grids).
template <bool BOUNDED, int LPC, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) fm_solve_kernel(FmSolveParams p, int it0, int it1) {
  if (*(volatile const int32_t*)(p.flags) != 0) return;  // the batch stopped at an earlier check
  __shared__ __align__(16) float smem[EPC * S_ELEM];
  __shared__ uint32_t jtab[36];
  if (threadIdx.x < 36) jtab[threadIdx.x] = kJacTable[threadIdx.x];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 4;
  const int64_t b = (int64_t)blockIdx.x * EPC + warp * EPW + g;
  if (b >= p.B) return;
  Group G{smem + (warp * EPW + g) * S_ELEM, 0xFFFFu << (g * GL), lane & 15, g * GL};
  const int l = G.l;
  const int T = p.T;
  const int nA = p.n_alpha;
  const int64_t rec_stride = (int64_t)(T + 1) * REC;
  float* slots = p.slots + b * (int64_t)(nA + 1) * rec_stride;
  float* kw = p.gains + b * (int64_t)T * KREC;
  float* fmw = p.free_mask + b * (int64_t)T * NUf;
  const float* xr = p.x_ref != nullptr ? p.x_ref + b * (int64_t)(T + 1) * NXf : nullptr;
  const float* ur = p.u_ref != nullptr ? p.u_ref + b * (int64_t)T * NUf : nullptr;
  const float* Cf = p.C_final != nullptr ? p.C_final + b * NN : nullptr;
  const float* cf = p.c_final != nullptr ? p.c_final + b * Nf : nullptr;
  const float* x0 = p.x0 + b * NXf;
  init_jacobian(G, p.dt);
  float ulo[4] = {0.0f, 0.0f, 0.0f, 0.0f}, uhi[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (BOUNDED) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ulo[i] = __ldg(p.u_min + i);
      uhi[i] = __ldg(p.u_max + i);
    }
  }
  const float* Cb = p.C + b * p.cost_bstride * NN;
  const float* cb = p.c + b * p.cost_bstride * Nf;
  auto Cstep = [&](int t) { return Cb + (int64_t)t * p.cost_tstride * NN; };
  auto cstep = [&](int t) { return cb + (int64_t)t * p.cost_tstride * Nf; };

  int nom = 0, lin = 0, code = 0;
  float best = 0.0f, imp = 0.0f;
  if (it0 == 0) {
    // trace rows start as "not run"; free masks as all free
    if (p.trace != nullptr)
      for (int i = l; i < p.max_iter; i += GL) p.trace[b * p.max_iter + i] = (int8_t)ILQR_TRACE_NOT_RUN;
    for (int i = l; i < T * NUf; i += GL) fmw[i] = 1.0f;
    // initial rollout of clamp(U_init) and its cost (compute_cost form): every
    // lane steps the same trajectory, the cost rows are split over the group
    {
      float x[10];
#pragma unroll
      for (int i = 0; i < 10; ++i) x[i] = __ldg(x0 + i);
      float total = 0.0f;
      for (int t = 0; t < T; ++t) {
        float u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float v = __ldg(p.U_init + (b * T + t) * NUf + i);
          u[i] = BOUNDED ? nan_clamp(v, ulo[i], uhi[i]) : v;
        }
        float* rec = slots + (int64_t)t * REC;
        float z[Nf];
#pragma unroll
        for (int i = 0; i < 10; ++i) {
          if (l == 0) rec[i] = x[i];
          z[i] = x[i] - (xr != nullptr ? xr[t * NXf + i] : 0.0f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (l == 0) rec[10 + i] = u[i];
          z[10 + i] = u[i] - (ur != nullptr ? ur[t * NUf + i] : 0.0f);
        }
        float qd, ln;
        quad_split<GL>(Cstep(t), cstep(t), z, l, G.gm, G.base, 0, qd, ln);
        total = total + (qd + ln);
        step_matrix(x, u, p.dt, x);
      }
      float* rec = slots + (int64_t)T * REC;
      float z[Nf];
#pragma unroll
      for (int i = 0; i < 10; ++i) {
        if (l == 0) rec[i] = x[i];
        z[i] = x[i] - (xr != nullptr ? xr[T * NXf + i] : 0.0f);
      }
#pragma unroll
      for (int i = 10; i < Nf; ++i) z[i] = 0.0f;
      float qd, ln;
      quad_split<GL>(Cf, cf, z, l, G.gm, G.base, 0, qd, ln);
      best = (total + qd) + ln;
    }
    nom = 0;
    lin = 0;
    code = 0;
  } else {
    nom = p.state.nom[b];
    lin = p.state.lin[b];
    best = p.state.best[b];
    code = p.state.code[b];
  }
  G.sync();

  for (int it = it0; it < it1; ++it) {
    if (code != 0) {
      // frozen: the same rejection again
      if (p.trace != nullptr && l == 0) p.trace[b * p.max_iter + it] = (int8_t)code;
      imp = best != best ? best : 0.0f;
      continue;
    }
    const float* nrec = slots + (int64_t)nom * rec_stride;
    // ---- Riccati pass at the nominal trajectory ----
    float Vr[NXf];
    {
      load_point(G, nrec + (int64_t)T * REC, xr != nullptr ? xr + T * NXf : nullptr, nullptr, true);
      if (l < NXf) {
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NXf; ++j) {
          const float cij = Cf != nullptr ? __ldg(Cf + l * Nf + j) : 0.0f;
          Vr[j] = cij;
          s = j == 0 ? cij * G.sm[S_EZ] : s + cij * G.sm[S_EZ + j];
        }
        G.sm[S_V + l] = s + (cf != nullptr ? __ldg(cf + l) : 0.0f);
      }
      G.sync();
    }
    for (int t = T - 1; t >= 0; --t) {
      load_point(G, nrec + (int64_t)t * REC, xr != nullptr ? xr + t * NXf : nullptr,
                 ur != nullptr ? ur + t * NUf : nullptr, false);
      jacobian(G, jtab, p.dt);
      float cx[Nf], cu[NUf], lxi = 0.0f, luj = 0.0f;
      cost_rows(G, Cstep(t), cstep(t), cx, lxi, cu, luj);
      riccati_step<BOUNDED ? 1 : 0>(G, Vr, cx, lxi, quu_entry(Cstep(t), l), luj, p.reg, p.u_min, p.u_max, nullptr,
                                    kw + (int64_t)t * KREC, BOUNDED ? fmw + t * NUf : nullptr);
    }
    // ---- line search: candidate a on lanes a*LPC .. a*LPC + LPC - 1 ----
    // (lanes past the last candidate repeat it without writing)
    float cost = 0.0f;
    {
      const int a_own = l / LPC;
      const int r = l % LPC;
      const bool writer = a_own < nA && r == 0;
      const int a = a_own < nA ? a_own : nA - 1;
      const float al = pick_alpha(p.alphas, a);
      const int slot = a < nom ? a : a + 1;
      float* crec = slots + (int64_t)slot * rec_stride;
      const int first = G.base + a_own * LPC;
      float x[10];
#pragma unroll
      for (int i = 0; i < 10; ++i) x[i] = __ldg(x0 + i);
      float total = 0.0f;
      for (int t = 0; t < T; ++t) {
        const float* nr = nrec + (int64_t)t * REC;
        const float* kr = kw + (int64_t)t * KREC;
        float dx[10], u[4], z[Nf];
#pragma unroll
        for (int i = 0; i < 10; ++i) dx[i] = x[i] - nr[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float du = al * kr[40 + i];
#pragma unroll
          for (int j = 0; j < 10; ++j) du = fmaf(kr[i * 10 + j], dx[j], du);
          const float v = nr[10 + i] + du;
          u[i] = BOUNDED ? fclamp(v, ulo[i], uhi[i]) : v;
        }
        float* rec = crec + (int64_t)t * REC;
#pragma unroll
        for (int i = 0; i < 10; ++i) {
          if (writer) rec[i] = x[i];
          z[i] = x[i] - (xr != nullptr ? xr[t * NXf + i] : 0.0f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (writer) rec[10 + i] = u[i];
          z[10 + i] = u[i] - (ur != nullptr ? ur[t * NUf + i] : 0.0f);
        }
        float qd, ln;
        quad_split<LPC>(Cstep(t), cstep(t), z, r, G.gm, first, 1, qd, ln);
        total = total + (qd + ln);
        step_cross(x, u, p.dt, x);
      }
      float* rec = crec + (int64_t)T * REC;
      float z[Nf];
#pragma unroll
      for (int i = 0; i < 10; ++i) {
        if (writer) rec[i] = x[i];
        z[i] = x[i] - (xr != nullptr ? xr[T * NXf + i] : 0.0f);
      }
#pragma unroll
      for (int i = 10; i < Nf; ++i) z[i] = 0.0f;
      float qd, ln;
      quad_split<LPC>(Cf, cf, z, r, G.gm, first, 1, qd, ln);
      cost = total + (qd + ln);
    }
    // ---- decision (lane 0 of the group) ----
    float cst[ILQR_MAX_ALPHAS_DEV];
#pragma unroll
    for (int a = 0; a < ILQR_MAX_ALPHAS_DEV; ++a) cst[a] = __shfl_sync(G.gm, cost, G.base + (a * LPC) % GL);
    // argmin over the step sizes: the first NaN if any (no improvement), else
    // the first minimum; improvement is strict (drone_ilqr_ext.cpp:1003-1022)
    int j = 0;
    bool improved;
    float newc;
    {
      int jnan = -1, jmin = -1;
      float cmin = 0.0f;
#pragma unroll
      for (int a = 0; a < ILQR_MAX_ALPHAS_DEV; ++a) {
        if (a < nA) {
          const float c = cst[a];
          if (c != c) {
            if (jnan < 0) jnan = a;
          } else if (jmin < 0 || c < cmin) {
            cmin = c;
            jmin = a;
          }
        }
      }
      j = jmin < 0 ? 0 : jmin;
      if (jnan >= 0) {
        j = jnan;
        improved = false;
        newc = best;
      } else {
        improved = cmin < best;
        newc = improved ? cmin : best;
      }
      if (p.forced != nullptr) {
        const int f = p.forced[b * p.max_iter + it];
        improved = f >= 0;
        j = improved ? f : -f - 1;
        float cj = cst[0];
#pragma unroll
        for (int a = 1; a < ILQR_MAX_ALPHAS_DEV; ++a) cj = (a == j) ? cst[a] : cj;
        newc = improved ? cj : best;
      }
    }
    const int tcode = improved ? j : -(j + 1);
    if (p.trace != nullptr && l == 0) p.trace[b * p.max_iter + it] = (int8_t)tcode;
    const float nb = improved ? newc : best;
    imp = fabsf(best - nb);
    lin = nom;
    if (improved) {
      nom = j < nom ? j : j + 1;
      best = nb;
    } else {
      code = tcode;
    }
    G.sync();
  }
  if (l == 0) {
    p.state.nom[b] = nom;
    p.state.lin[b] = lin;
    p.state.best[b] = best;
    p.state.code[b] = code;
    p.state.imp[b] = imp;
  }
}

// After a segment ending at iteration `it_end` (a check iteration): the
// batch maximum of the last improvements (NaN if any is NaN) against the
// tolerance (drone_ilqr_ext.cpp:1029-1049), or the forced stop.
__global__ void __launch_bounds__(1024) fm_check_kernel(FmSolveParams p, int it_end) {
  __shared__ float red[32];
  __shared__ int nan_seen;
  if (*(volatile const int32_t*)(p.flags) != 0) return;
  if (threadIdx.x == 0) nan_seen = 0;
  __syncthreads();
  float m = 0.0f;
  bool nan = false;
  for (int64_t b = threadIdx.x; b < p.B; b += blockDim.x) {
    const float v = p.state.imp[b];
    if (v != v) nan = true;
    else m = fmaxf(m, v);
  }
  if (nan) atomicOr(&nan_seen, 1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    const bool conv = !nan_seen && (double)mx < (double)p.tol;
    const bool last = it_end >= p.max_iter;
    bool stop = conv;
    if (p.forced_stop > 0 && !last) stop = it_end == p.forced_stop;
    p.flags[2] = it_end;
    if (last) {
      p.flags[1] = conv ? 1 : 0;
    } else if (stop) {
      p.flags[1] = 1;
      p.flags[0] = 1;
    }
  }
}

// Outputs: X, U from the nominal slot, X_lin, U_lin from the linearisation
// slot, tight = free mask < 0.5 (drone_ilqr_ext.cpp:1052-1061).
__global__ void __launch_bounds__(256) fm_finalize_kernel(FmSolveParams p) {
  const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (b >= p.B) return;
  const int T = p.T;
  const int64_t rec_stride = (int64_t)(T + 1) * REC;
  const float* slots = p.slots + b * (int64_t)(p.n_alpha + 1) * rec_stride;
  const int nom = p.max_iter > 0 ? p.state.nom[b] : 0;
  const int lin = p.max_iter > 0 ? p.state.lin[b] : 0;
  const float* nr = slots + (int64_t)nom * rec_stride;
  const float* lr = slots + (int64_t)lin * rec_stride;
  for (int i = l; i < (T + 1) * NXf; i += 32) {
    const int t = i / NXf, k = i % NXf;
    p.X[b * (int64_t)(T + 1) * NXf + i] = nr[(int64_t)t * REC + k];
    if (p.X_lin != nullptr) p.X_lin[b * (int64_t)(T + 1) * NXf + i] = lr[(int64_t)t * REC + k];
  }
  for (int i = l; i < T * NUf; i += 32) {
    const int t = i / NUf, k = i % NUf;
    p.U[b * (int64_t)T * NUf + i] = nr[(int64_t)t * REC + NXf + k];
    if (p.U_lin != nullptr) p.U_lin[b * (int64_t)T * NUf + i] = lr[(int64_t)t * REC + NXf + k];
    if (p.tight != nullptr) {
      const bool bounded = p.u_min != nullptr && p.u_max != nullptr;
      p.tight[b * (int64_t)T * NUf + i] = (bounded && p.free_mask[b * (int64_t)T * NUf + i] < 0.5f) ? 1 : 0;
    }
  }
  if (l == 0 && p.best_cost != nullptr) p.best_cost[b] = p.max_iter > 0 ? p.state.best[b] : 0.0f;
}

// ---------------------------------------------------------------------------
// Backward: masked adjoint Riccati, tangent sweep, gradients
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(THREADS, 4) fm_backward_kernel(FmBackwardParams p) {
  __shared__ __align__(16) float smem[EPC * S_ELEM];
  __shared__ uint32_t jtab[36];
  if (threadIdx.x < 36) jtab[threadIdx.x] = kJacTable[threadIdx.x];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 4;
  const int64_t b = (int64_t)blockIdx.x * EPC + warp * EPW + g;
  if (b >= p.B) return;
  Group G{smem + (warp * EPW + g) * S_ELEM, 0xFFFFu << (g * GL), lane & 15, g * GL};
  float* sm = G.sm;
  const int l = G.l;
  const int T = p.T;
  float* kw = p.gains + b * (int64_t)T * KREC;
  const float* Xl = p.X_lin + b * (int64_t)(T + 1) * NXf;
  const float* Ul = p.U_lin + b * (int64_t)T * NUf;
  const float* X = p.X + b * (int64_t)(T + 1) * NXf;
  const float* U = p.U + b * (int64_t)T * NUf;
  const float* gX = p.grad_X + b * (int64_t)(T + 1) * NXf;
  const float* gU = p.grad_U + b * (int64_t)T * NUf;
  const float* xr = p.x_ref != nullptr ? p.x_ref + b * (int64_t)(T + 1) * NXf : nullptr;
  const float* ur = p.u_ref != nullptr ? p.u_ref + b * (int64_t)T * NUf : nullptr;
  const float* Cf = p.C_final != nullptr ? p.C_final + b * NN : nullptr;
  const float* Cb = p.C + b * p.cost_bstride * NN;
  init_jacobian(G, p.dt);
  auto load_lin = [&](int t) {
    if (l < NXf) sm[S_Z + l] = Xl[t * NXf + l];
    else if (l < Nf) sm[S_Z + l] = Ul[t * NUf + l - NXf];
    G.sync();
  };
  // terminal: V = C_f[:10,:10], v = -dL/dX_T
  float Vr[NXf];
  if (l < NXf) {
#pragma unroll
    for (int j = 0; j < NXf; ++j) Vr[j] = Cf != nullptr ? __ldg(Cf + l * Nf + j) : 0.0f;
    sm[S_V + l] = -gX[T * NXf + l];
  }
  G.sync();
  for (int t = T - 1; t >= 0; --t) {
    load_lin(t);
    jacobian(G, jtab, p.dt);
    const float* cs = Cb + (int64_t)t * p.cost_tstride * NN;
    float cx[Nf], lxi = 0.0f, luj = 0.0f;
    if (l < NXf) {
#pragma unroll
      for (int j = 0; j < Nf; ++j) cx[j] = __ldg(cs + l * Nf + j);
      lxi = -gX[t * NXf + l];
    } else if (l < Nf) {
      luj = -gU[t * NUf + l - NXf];
    }
    const float cq = quu_entry(cs, l);
    if (p.tight != nullptr) {
      riccati_step<2>(G, Vr, cx, lxi, cq, luj, p.reg, nullptr, nullptr, p.tight + (b * (int64_t)T + t) * NUf,
                      kw + (int64_t)t * KREC, nullptr);
    } else {
      riccati_step<0>(G, Vr, cx, lxi, cq, luj, p.reg, nullptr, nullptr, nullptr, kw + (int64_t)t * KREC, nullptr);
    }
  }
  if (p.grad_x0 != nullptr && l < NXf) p.grad_x0[b * NXf + l] = -sm[S_V + l];
  // tangent sweep (backward_pass_kernel.cu:1146-1212)
  if (l < NXf) sm[S_DX + l] = 0.0f;
  G.sync();
  float* gC = p.grad_C != nullptr ? p.grad_C + b * p.cost_bstride * NN : nullptr;
  float* gc = p.grad_c != nullptr ? p.grad_c + b * p.cost_bstride * Nf : nullptr;
  for (int t = 0; t < T; ++t) {
    load_lin(t);
    jacobian(G, jtab, p.dt);
    const float* kr = kw + (int64_t)t * KREC;
    if (l < NUf) {
      float s = kr[40 + l];
#pragma unroll
      for (int j = 0; j < NXf; ++j) s = fmaf(kr[l * 10 + j], sm[S_DX + j], s);
      sm[S_DU + l] = s;
    }
    // tau = [X_t - x_ref_t; U_t - u_ref_t] at the solution, into S_EZ
    if (l < NXf) sm[S_EZ + l] = X[t * NXf + l] - (xr != nullptr ? xr[t * NXf + l] : 0.0f);
    else if (l < Nf) sm[S_EZ + l] = U[t * NUf + l - NXf] - (ur != nullptr ? ur[t * NUf + l - NXf] : 0.0f);
    G.sync();
    float dxn = 0.0f;
    if (l < NXf) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < NXf; ++j) s = fmaf(sm[S_A + l * 10 + j], sm[S_DX + j], s);
#pragma unroll
      for (int j = 0; j < NUf; ++j) s = fmaf(sm[S_B + l * 4 + j], sm[S_DU + j], s);
      dxn = s;
    }
    if (l < Nf) {
      // d_tau = [dX_t; dU_t] occupies S_DX..S_DU contiguously
      const float dti = sm[S_DX + l];
      const float ti = sm[S_EZ + l];
      if (gC != nullptr) {
        float* row = gC + (int64_t)t * p.cost_tstride * NN + l * Nf;
#pragma unroll
        for (int j = 0; j < Nf; ++j) row[j] = -0.5f * (dti * sm[S_EZ + j] + ti * sm[S_DX + j]);
      }
      if (gc != nullptr) gc[(int64_t)t * p.cost_tstride * Nf + l] = -dti;
      if (l < NXf && p.grad_x_ref != nullptr) p.grad_x_ref[(b * (int64_t)(T + 1) + t) * NXf + l] = dti;
      if (l >= NXf && p.grad_u_ref != nullptr) p.grad_u_ref[(b * (int64_t)T + t) * NUf + l - NXf] = dti;
    }
    G.sync();
    if (l < NXf) sm[S_DX + l] = dxn;
    G.sync();
  }
  // terminal gradients: tau_N = [X_T - x_ref_T; 0], d tau_N = [dX_T; 0]
  const float dti = l < NXf ? sm[S_DX + l] : 0.0f;
  const float ti = l < NXf ? X[T * NXf + l] - (xr != nullptr ? xr[T * NXf + l] : 0.0f) : 0.0f;
  if (l < Nf) sm[S_EZ + l] = ti;
  G.sync();
  if (l < Nf) {
    if (l < NXf && p.grad_x_ref != nullptr) p.grad_x_ref[(b * (int64_t)(T + 1) + T) * NXf + l] = dti;
    if (p.grad_c_final != nullptr) p.grad_c_final[b * Nf + l] = -dti;
    if (p.grad_C_final != nullptr) {
#pragma unroll
      for (int j = 0; j < Nf; ++j) {
        const float dtj = j < NXf ? sm[S_DX + j] : 0.0f;
        p.grad_C_final[b * NN + l * Nf + j] = -0.5f * (dti * sm[S_EZ + j] + ti * dtj);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Extension-surface kernels: the reference extension's separate entry points
// with its numerics, one thread per step or per element (a compatibility
// path; the solve and backward above are the fused ones)
// ---------------------------------------------------------------------------

// A [n][10][10], B [n][10][4] at the points (X[b][t], U[b][t]), t < T
// (drone_kernels.cu:64-190), with the entry values of the fused kernels.
__global__ void fm_linearize_kernel(const float* __restrict__ X, const float* __restrict__ U, int64_t B, int T,
                                    float dt, float* __restrict__ A, float* __restrict__ Bm) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int64_t b = i / T;
  const int t = (int)(i - b * T);
  const float* x = X + (b * (T + 1) + t) * NXf;
  const float* u = U + i * NUf;
  float* Ai = A + i * NXf * NXf;
  float* Bi = Bm + i * NXf * NUf;
  for (int e = 0; e < NXf * NXf; ++e) {
    const int r = e / NXf, c = e % NXf;
    float v = r == c ? 1.0f : 0.0f;
    if ((r == 0 && c == 7) || (r == 1 && c == 8) || (r == 2 && c == 9)) v = dt;
    Ai[e] = v;
  }
  for (int e = 0; e < NXf * NUf; ++e) Bi[e] = 0.0f;
  const float fc = u[0];
  const float fcm = fc / MASS;
  float var[11];
  for (int l = 0; l < 3; ++l) var[l] = u[1 + l];
  for (int l = 3; l < 7; ++l) var[l] = x[l];
  for (int l = 7; l < 11; ++l) var[l] = x[l - 4] * fcm;
  const float h = 0.5f * dt, t2 = 2.0f * dt;
  for (int e = 0; e < 36; ++e) {
    const uint32_t code = kJacTable[e];
    const float p = (((code >> 13) & 1u) ? t2 : h) * var[(code >> 9) & 15u];
    const bool minus = (code >> 15) & 1u;
    const float v = ((code >> 14) & 1u) == 0u ? (minus ? 0.0f - p : 0.0f + p) : (minus ? -p : p);
    const uint32_t dst = code & 511u;  // offset in the shared-memory block: A at S_A, B at S_B
    if (dst < (uint32_t)S_B) Ai[dst - S_A] = v;
    else Bi[dst - S_B] = v;
  }
  const float qw = x[3], qx = x[4], qy = x[5], qz = x[6];
  const float dtm = dt / MASS;
  Bi[7 * NUf] = 2.0f * (qx * qz + qw * qy) * dtm;
  Bi[8 * NUf] = 2.0f * (qy * qz - qw * qx) * dtm;
  Bi[9 * NUf] = (qw * qw - qx * qx - qy * qy + qz * qz) * dtm;
}

// drone_backward_pass_batched on given matrices (backward_pass_kernel.cu:
// 617-745): Q terms with reg once; a tight control's row and column of Q_uu
// are zeroed with a 1e-11 diagonal, its column of Q_xu and entry of q_u
// zeroed; gains by the pivoted LU; V = Q_xx + Q_xu K, v = q_x + Q_xu k.
__global__ void fm_adjoint_lqr_kernel(const float* __restrict__ A, const float* __restrict__ Bm,
                                      const float* __restrict__ l_xx, const float* __restrict__ l_uu,
                                      const float* __restrict__ l_xu, const float* __restrict__ l_x,
                                      const float* __restrict__ l_u, const float* __restrict__ l_xxN,
                                      const float* __restrict__ l_xN, const uint8_t* __restrict__ tight, int64_t B,
                                      int T, float reg, float* __restrict__ Kout, float* __restrict__ kout,
                                      float* __restrict__ v0) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float V[NXf][NXf], v[NXf];
  for (int i = 0; i < NXf; ++i) {
    v[i] = l_xN[b * NXf + i];
    for (int j = 0; j < NXf; ++j) V[i][j] = l_xxN[(b * NXf + i) * NXf + j];
  }
  for (int t = T - 1; t >= 0; --t) {
    const int64_t bt = b * T + t;
    const float* At = A + bt * NXf * NXf;
    const float* Bt = Bm + bt * NXf * NUf;
    float VA[NXf][NXf], VB[NXf][NUf];
    for (int i = 0; i < NXf; ++i) {
      for (int j = 0; j < NXf; ++j) {
        float s = 0.0f;
        for (int k = 0; k < NXf; ++k) s = fmaf(V[i][k], At[k * NXf + j], s);
        VA[i][j] = s;
      }
      for (int j = 0; j < NUf; ++j) {
        float s = 0.0f;
        for (int k = 0; k < NXf; ++k) s = fmaf(V[i][k], Bt[k * NUf + j], s);
        VB[i][j] = s;
      }
    }
    float Qxx[NXf][NXf], Qxu[NXf][NUf], qx[NXf], H[4][4], q[4];
    for (int i = 0; i < NXf; ++i) {
      for (int j = 0; j < NXf; ++j) {
        float s = l_xx[bt * NXf * NXf + i * NXf + j];
        for (int k = 0; k < NXf; ++k) s = fmaf(At[k * NXf + i], VA[k][j], s);
        Qxx[i][j] = s;
      }
      for (int j = 0; j < NUf; ++j) {
        float s = l_xu[bt * NXf * NUf + i * NUf + j];
        for (int k = 0; k < NXf; ++k) s = fmaf(At[k * NXf + i], VB[k][j], s);
        Qxu[i][j] = s;
      }
      float s = l_x[bt * NXf + i];
      for (int k = 0; k < NXf; ++k) s = fmaf(At[k * NXf + i], v[k], s);
      qx[i] = s;
    }
    for (int a = 0; a < NUf; ++a) {
      for (int c = 0; c < NUf; ++c) {
        float s = l_uu[bt * NUf * NUf + a * NUf + c];
        for (int k = 0; k < NXf; ++k) s = fmaf(Bt[k * NUf + a], VB[k][c], s);
        if (a == c) s = s + reg;
        H[a][c] = s;
      }
      float s = l_u[bt * NUf + a];
      for (int k = 0; k < NXf; ++k) s = fmaf(Bt[k * NUf + a], v[k], s);
      q[a] = s;
    }
    if (tight != nullptr) {
      float fr[4];
      for (int a = 0; a < NUf; ++a) fr[a] = tight[bt * NUf + a] ? 0.0f : 1.0f;
      for (int a = 0; a < NUf; ++a) {
        for (int c = 0; c < NUf; ++c) H[a][c] = H[a][c] * (fr[a] * fr[c]);
        if (fr[a] == 0.0f) H[a][a] = H[a][a] + 1e-11f;
        q[a] = q[a] * fr[a];
        for (int r = 0; r < NXf; ++r) Qxu[r][a] = Qxu[r][a] * fr[a];
      }
    }
    int piv[4];
    lu_factor4(H, piv);
    float K[NUf][NXf], kk[4];
    for (int j = 0; j < NXf; ++j) {
      float rhs[4];
      for (int a = 0; a < NUf; ++a) rhs[a] = -Qxu[j][a];
      lu_solve4(H, piv, rhs);
      for (int a = 0; a < NUf; ++a) K[a][j] = rhs[a];
    }
    for (int a = 0; a < NUf; ++a) kk[a] = -q[a];
    lu_solve4(H, piv, kk);
    for (int a = 0; a < NUf; ++a) {
      for (int j = 0; j < NXf; ++j) Kout[(bt * NUf + a) * NXf + j] = K[a][j];
      kout[bt * NUf + a] = kk[a];
    }
    for (int i = 0; i < NXf; ++i) {
      for (int j = 0; j < NXf; ++j) {
        float s = Qxx[i][j];
        for (int m = 0; m < NUf; ++m) s = fmaf(Qxu[i][m], K[m][j], s);
        V[i][j] = s;
      }
      float s = qx[i];
      for (int m = 0; m < NUf; ++m) s = fmaf(Qxu[i][m], kk[m], s);
      v[i] = s;
    }
  }
  for (int i = 0; i < NXf; ++i) v0[b * NXf + i] = v[i];
}

// drone_implicit_diff_assembly (backward_pass_kernel.cu:1092-1256): the
// tangent sweep dU = K dX + k, dX' = A dX + B dU from dX_0 = 0, then
// grad_C = -1/2 (d tau tau^T + tau d tau^T), grad_c = -d tau with
// tau = [X - x_ref; U - u_ref], grad_x_ref = dX (t = 0..T), grad_u_ref = dU,
// grad_x0 = -v0, and the terminal grad_C_final, grad_c_final. Outputs may be
// null except grad_C, grad_c, grad_x0.
__global__ void fm_assembly_kernel(const float* __restrict__ K, const float* __restrict__ k,
                                   const float* __restrict__ v0, const float* __restrict__ A,
                                   const float* __restrict__ Bm, const float* __restrict__ X,
                                   const float* __restrict__ U, const float* __restrict__ x_ref,
                                   const float* __restrict__ u_ref, int64_t B, int T, float* gC, float* gc,
                                   float* gx0, float* gxr, float* gur, float* gCf, float* gcf) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  for (int i = 0; i < NXf; ++i) gx0[b * NXf + i] = -v0[b * NXf + i];
  float dX[NXf];
  for (int i = 0; i < NXf; ++i) dX[i] = 0.0f;
  for (int t = 0; t < T; ++t) {
    const int64_t bt = b * T + t;
    float dU[NUf], tau[Nf], dt_[Nf];
    for (int a = 0; a < NUf; ++a) {
      float s = k[bt * NUf + a];
      for (int j = 0; j < NXf; ++j) s = fmaf(K[(bt * NUf + a) * NXf + j], dX[j], s);
      dU[a] = s;
    }
    for (int i = 0; i < NXf; ++i) {
      tau[i] = X[(b * (T + 1) + t) * NXf + i] - (x_ref != nullptr ? x_ref[(b * (T + 1) + t) * NXf + i] : 0.0f);
      dt_[i] = dX[i];
    }
    for (int a = 0; a < NUf; ++a) {
      tau[NXf + a] = U[bt * NUf + a] - (u_ref != nullptr ? u_ref[bt * NUf + a] : 0.0f);
      dt_[NXf + a] = dU[a];
    }
    for (int i = 0; i < Nf; ++i) {
      for (int j = 0; j < Nf; ++j) gC[(bt * Nf + i) * Nf + j] = -0.5f * (dt_[i] * tau[j] + tau[i] * dt_[j]);
      gc[bt * Nf + i] = -dt_[i];
    }
    if (gxr != nullptr)
      for (int i = 0; i < NXf; ++i) gxr[(b * (T + 1) + t) * NXf + i] = dX[i];
    if (gur != nullptr)
      for (int a = 0; a < NUf; ++a) gur[bt * NUf + a] = dU[a];
    float dn[NXf];
    for (int i = 0; i < NXf; ++i) {
      float s = 0.0f;
      for (int j = 0; j < NXf; ++j) s = fmaf(A[(bt * NXf + i) * NXf + j], dX[j], s);
      for (int j = 0; j < NUf; ++j) s = fmaf(Bm[(bt * NXf + i) * NUf + j], dU[j], s);
      dn[i] = s;
    }
    for (int i = 0; i < NXf; ++i) dX[i] = dn[i];
  }
  if (gxr != nullptr)
    for (int i = 0; i < NXf; ++i) gxr[(b * (T + 1) + T) * NXf + i] = dX[i];
  float tn[Nf], dn[Nf];
  for (int i = 0; i < Nf; ++i) {
    tn[i] = i < NXf ? X[(b * (T + 1) + T) * NXf + i] - (x_ref != nullptr ? x_ref[(b * (T + 1) + T) * NXf + i] : 0.0f)
                    : 0.0f;
    dn[i] = i < NXf ? dX[i] : 0.0f;
  }
  if (gCf != nullptr)
    for (int i = 0; i < Nf; ++i)
      for (int j = 0; j < Nf; ++j) gCf[(b * Nf + i) * Nf + j] = -0.5f * (dn[i] * tn[j] + tn[i] * dn[j]);
  if (gcf != nullptr)
    for (int i = 0; i < Nf; ++i) gcf[b * Nf + i] = -dn[i];
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

cudaError_t launch_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A, float* Bm,
                             cudaStream_t stream) {
  const int64_t n = B * T;
  if (n == 0) return cudaSuccess;
  fm_linearize_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(X, U, B, T, dt, A, Bm);
  return cudaGetLastError();
}

cudaError_t launch_adjoint_lqr(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                               const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                               const float* l_xN, const uint8_t* tight, int64_t B, int T, float reg, float* K,
                               float* k, float* v0, cudaStream_t stream) {
  if (B == 0) return cudaSuccess;
  fm_adjoint_lqr_kernel<<<(unsigned)((B + 63) / 64), 64, 0, stream>>>(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN,
                                                                      l_xN, tight, B, T, reg, K, k, v0);
  return cudaGetLastError();
}

cudaError_t launch_assembly(const float* K, const float* k, const float* v0, const float* A, const float* Bm,
                            const float* X, const float* U, const float* x_ref, const float* u_ref, int64_t B,
                            int T, float* gC, float* gc, float* gx0, float* gxr, float* gur, float* gCf, float* gcf,
                            cudaStream_t stream) {
  if (B == 0) return cudaSuccess;
  fm_assembly_kernel<<<(unsigned)((B + 63) / 64), 64, 0, stream>>>(K, k, v0, A, Bm, X, U, x_ref, u_ref, B, T, gC,
                                                                   gc, gx0, gxr, gur, gCf, gcf);
  return cudaGetLastError();
}


size_t solve_ws_bytes(int64_t B, int32_t T, int32_t n_alpha) {
  const size_t slots = (size_t)B * (n_alpha + 1) * (T + 1) * REC * sizeof(float);
  const size_t gains = (size_t)B * T * KREC * sizeof(float);
  const size_t fm = (size_t)B * T * NUf * sizeof(float);
  const size_t st = (size_t)B * 5 * sizeof(int32_t);
  return 256 + slots + gains + fm + st;
}

size_t backward_ws_bytes(int64_t B, int32_t T) { return 256 + (size_t)B * T * KREC * sizeof(float); }

void carve_solve(FmSolveParams& p, void* ws) {
  char* w = static_cast<char*>(ws);
  p.flags = reinterpret_cast<int32_t*>(w);
  w += 256;
  p.slots = reinterpret_cast<float*>(w);
  w += (size_t)p.B * (p.n_alpha + 1) * (p.T + 1) * REC * sizeof(float);
  p.gains = reinterpret_cast<float*>(w);
  w += (size_t)p.B * p.T * KREC * sizeof(float);
  p.free_mask = reinterpret_cast<float*>(w);
  w += (size_t)p.B * p.T * NUf * sizeof(float);
  p.state.nom = reinterpret_cast<int32_t*>(w);
  p.state.lin = p.state.nom + p.B;
  p.state.code = p.state.lin + p.B;
  p.state.best = reinterpret_cast<float*>(p.state.code + p.B);
  p.state.imp = p.state.best + p.B;
}

// One solve segment in the register tier chosen by the caller.
template <bool BOUNDED, int LPC>
void launch_segment(const FmSolveParams& p, unsigned grid, bool fat, int it0, int it1, cudaStream_t stream) {
  if (fat) fm_solve_kernel<BOUNDED, LPC, 2><<<grid, THREADS, 0, stream>>>(p, it0, it1);
  else fm_solve_kernel<BOUNDED, LPC, 3><<<grid, THREADS, 0, stream>>>(p, it0, it1);
}

cudaError_t launch_solve(FmSolveParams& p, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.flags, 0, 256, stream);
  if (e != cudaSuccess || p.B == 0) return e;
  const unsigned grid = (unsigned)((p.B + EPC - 1) / EPC);
  const bool bounded = p.u_min != nullptr && p.u_max != nullptr;
  const int segs = p.max_iter > 0 ? (p.max_iter + FM_CHECK_PERIOD - 1) / FM_CHECK_PERIOD : 1;
  for (int s = 0; s < segs; ++s) {
    const int it0 = s * FM_CHECK_PERIOD;
    const int it1 = p.max_iter > 0 ? (it0 + FM_CHECK_PERIOD < p.max_iter ? it0 + FM_CHECK_PERIOD : p.max_iter) : 0;
    const bool wide = p.n_alpha <= GL / 4;
    // one wave at 2 CTAs per SM runs the fat tier (B = 2048: 0.89 against
    // 1.01 ms at 4 CTAs per SM); larger grids the 3-CTA tier (B = 16384: 5.35
    // ms, against 5.45 ms at 4 and 6.22 ms at 2)
    const bool fat = grid <= 2u * SM_COUNT_FM;
    if (bounded) {
      if (wide) launch_segment<true, 4>(p, grid, fat, it0, it1, stream);
      else launch_segment<true, 2>(p, grid, fat, it0, it1, stream);
    } else {
      if (wide) launch_segment<false, 4>(p, grid, fat, it0, it1, stream);
      else launch_segment<false, 2>(p, grid, fat, it0, it1, stream);
    }
    if (p.max_iter > 0) fm_check_kernel<<<1, 1024, 0, stream>>>(p, it1);
  }
  const unsigned fgrid = (unsigned)((p.B + 7) / 8);
  fm_finalize_kernel<<<fgrid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_backward(FmBackwardParams& p, cudaStream_t stream) {
  if (p.B == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((p.B + EPC - 1) / EPC);
  fm_backward_kernel<<<grid, THREADS, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace fm
}  // namespace ilqr
