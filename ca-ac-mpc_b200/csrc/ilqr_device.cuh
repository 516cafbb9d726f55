// ilqr_device.cuh -- device building blocks of the B200 iLQR solver.
//
// Compiled with -fmad=false: a*b+c is never contracted implicitly, so the
// model arithmetic follows the reference's torch elementwise ops term by term
// (divisions by the mass and the normalisation of the body rates are
// multiplications by reciprocals, within 1 ulp of a division), and the linear
// algebra uses explicit fmaf() with a fixed summation order (deterministic: a
// recomputed rollout is bit-identical to the candidate it repeats).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ilqr {

constexpr int NX = 10;
constexpr int NU = 4;
constexpr int NT = 14;              // NX + NU
constexpr int CBLK = NT * NT;       // floats of one C[b,t] block
constexpr int WARP = 32;            // threads per CTA (one warp)
constexpr float MASS = 0.752f;      // drone.py:166
constexpr float GZ = -9.8066f;      // drone.py:187
constexpr unsigned FULL = 0xffffffffu;
constexpr uint32_t WAIT_LIMIT = 1u << 24;   // bounded mbarrier polls

// Status bits (mirror ilqr_b200.h).
constexpr uint32_t ELEM_CHOL_FALLBACK = 1u;
constexpr uint32_t ELEM_NONFINITE = 2u;
constexpr uint32_t ELEM_PIPE_TIMEOUT = 4u;
constexpr uint32_t ELEM_DIAG_COST = 8u;

// --------------------------------------------------------------------------
// Quadrotor CTBR model (acmpc_public-master/diff_mpc_drones/drone.py)
// --------------------------------------------------------------------------

// One Euler/exp-map step, DroneDx.forward_CTBR (drone.py:409-465). The
// expressions follow drone.py's operation order term by term (quat_mult at
// :28-33, exp_map at :18-26, rotate_quat at :145-156); the zero terms of
// quat_mult(q, [0,0,0,fc]) contribute exact zeros and are elided.
__device__ __forceinline__ void drone_step(const float (&x)[NX], const float (&u)[NU],
                                           float dt, float (&xn)[NX]) {
  const float q0 = x[3], q1 = x[4], q2 = x[5], q3 = x[6];
  const float wx = u[1], wy = u[2], wz = u[3], fc = u[0];
  // p+ = p + dt v
  xn[0] = x[0] + dt * x[7];
  xn[1] = x[1] + dt * x[8];
  xn[2] = x[2] + dt * x[9];
  // exp_map(w, dt): torch.norm, F.normalize (eps 1e-12), cos/sin(|w| dt/2);
  // the three quotients use one correctly rounded reciprocal
  const float wn = sqrtf((wx * wx + wy * wy) + wz * wz);
  const float rden = __frcp_rn(fmaxf(wn, 1e-12f));
  const float nx = wx * rden, ny = wy * rden, nz = wz * rden;
  const float half = wn * (dt * 0.5f);
  float s, co;
  sincosf(half, &s, &co);
  const float e0 = co, e1 = nx * s, e2 = ny * s, e3 = nz * s;
  // q+ = quat_mult(q, em): q1 := q, q2 := em
  xn[3] = ((e0 * q0 - e1 * q1) - e2 * q2) - e3 * q3;
  xn[4] = ((e0 * q1 + e1 * q0) - e2 * q3) + e3 * q2;
  xn[5] = ((e0 * q2 + e2 * q0) + e1 * q3) - e3 * q1;
  xn[6] = ((e0 * q3 - e1 * q2) + e2 * q1) + e3 * q0;
  // rotate_quat(q, [0,0,fc]) = Im( (q (x) [0,0,0,fc]) (x) conj(q) )
  const float f0 = -(fc * q3), f1 = fc * q2, f2 = -(fc * q1), f3 = fc * q0;
  const float c1 = -q1, c2 = -q2, c3 = -q3;
  const float r1 = ((q0 * f1 + c1 * f0) - c2 * f3) + c3 * f2;
  const float r2 = ((q0 * f2 + c2 * f0) + c1 * f3) - c3 * f1;
  const float r3 = ((q0 * f3 - c1 * f2) + c2 * f1) + c3 * f0;
  // v+ = v + dt (rot/m + g), rot/m as rot * (1/m)
  constexpr float INV_MASS = 1.0f / MASS;
  xn[7] = x[7] + dt * (r1 * INV_MASS + 0.0f);
  xn[8] = x[8] + dt * (r2 * INV_MASS + 0.0f);
  xn[9] = x[9] + dt * (r3 * INV_MASS + GZ);
}

// Nonzero entries of the discrete Jacobians A = I + dt J_x, B = dt J_u
// (DroneDx.grad_input / get_A_B_mat_CTBR, drone.py:489-540). With state
// blocks p = 0..2, q = 3..6, v = 7..9 and controls (fc, wx, wy, wz):
//   A[p_i][v_i] = dt
//   A[q][q]  = [[1,-h0,-h1,-h2],[h0,1,h2,-h1],[h1,-h2,1,h0],[h2,h1,-h0,1]]
//   A[v][q]  = [[g2,g3,g0,g1],[-g1,-g0,g3,g2],[g0,-g1,-g2,g3]]
//   B[q][w]  = rows [-e1,-e2,-e3],[e0,-e3,-e2],[e3,e0,-e1],[-e2,e1,e0]
//   B[v][fc] = bv
// with h_k = (w_k/2) dt, g_i = 2 (q_i fc / m) dt, e_i = (q_i/2) dt,
// bv = (q^T M_k q / m) dt. All other entries are 0 (diagonal 1 for A).
struct Jac {
  float dt, h0, h1, h2, g0, g1, g2, g3, e0, e1, e2, e3, bv0, bv1, bv2;
};

__device__ __forceinline__ Jac drone_jac(const float (&x)[NX], const float (&u)[NU], float dt) {
  Jac J;
  J.dt = dt;
  J.h0 = (0.5f * u[1]) * dt;
  J.h1 = (0.5f * u[2]) * dt;
  J.h2 = (0.5f * u[3]) * dt;
  // The linearisation multiplies by 1/m (within 1 ulp of the reference's
  // division; the dynamics step itself keeps the division).
  constexpr float INV_MASS = 1.0f / MASS;
  const float a0 = x[3], a1 = x[4], a2 = x[5], a3 = x[6], fc = u[0];
  J.g0 = (2.0f * ((a0 * fc) * INV_MASS)) * dt;
  J.g1 = (2.0f * ((a1 * fc) * INV_MASS)) * dt;
  J.g2 = (2.0f * ((a2 * fc) * INV_MASS)) * dt;
  J.g3 = (2.0f * ((a3 * fc) * INV_MASS)) * dt;
  J.e0 = (0.5f * a0) * dt;
  J.e1 = (0.5f * a1) * dt;
  J.e2 = (0.5f * a2) * dt;
  J.e3 = (0.5f * a3) * dt;
  const float d1 = ((a2 * a0 + a3 * a1) + a0 * a2) + a1 * a3;
  const float d2 = ((-a1 * a0 + -a0 * a1) + a3 * a2) + a2 * a3;
  const float d3 = ((a0 * a0 + -a1 * a1) + -a2 * a2) + a3 * a3;
  J.bv0 = (d1 * INV_MASS) * dt;
  J.bv1 = (d2 * INV_MASS) * dt;
  J.bv2 = (d3 * INV_MASS) * dt;
  return J;
}

// A[q_m][q_j]
__device__ __forceinline__ float aqq(const Jac& J, int m, int j) {
  switch (m * 4 + j) {
    case 0: return 1.0f;   case 1: return -J.h0;  case 2: return -J.h1;  case 3: return -J.h2;
    case 4: return J.h0;   case 5: return 1.0f;   case 6: return J.h2;   case 7: return -J.h1;
    case 8: return J.h1;   case 9: return -J.h2;  case 10: return 1.0f;  case 11: return J.h0;
    case 12: return J.h2;  case 13: return J.h1;  case 14: return -J.h0; default: return 1.0f;
  }
}
// A[v_n][q_j]
__device__ __forceinline__ float avq(const Jac& J, int n, int j) {
  switch (n * 4 + j) {
    case 0: return J.g2;   case 1: return J.g3;   case 2: return J.g0;   case 3: return J.g1;
    case 4: return -J.g1;  case 5: return -J.g0;  case 6: return J.g3;   case 7: return J.g2;
    case 8: return J.g0;   case 9: return -J.g1;  case 10: return -J.g2; default: return J.g3;
  }
}
// B[q_m][w_k]
__device__ __forceinline__ float bqw(const Jac& J, int m, int k) {
  switch (m * 3 + k) {
    case 0: return -J.e1;  case 1: return -J.e2;  case 2: return -J.e3;
    case 3: return J.e0;   case 4: return -J.e3;  case 5: return -J.e2;
    case 6: return J.e3;   case 7: return J.e0;   case 8: return -J.e1;
    case 9: return -J.e2;  case 10: return J.e1;  default: return J.e0;
  }
}
__device__ __forceinline__ float bvf(const Jac& J, int n) {
  return n == 0 ? J.bv0 : (n == 1 ? J.bv1 : J.bv2);
}

// y = A x (sparse), the forward sweep / tangent step.
__device__ __forceinline__ void jac_apply(const Jac& J, const float (&x)[NX], const float (&u)[NU],
                                          float (&y)[NX]) {
#pragma unroll
  for (int i = 0; i < 3; ++i) y[i] = fmaf(J.dt, x[7 + i], x[i]);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = fmaf(aqq(J, m, j), x[3 + j], acc);
#pragma unroll
    for (int k = 0; k < 3; ++k) acc = fmaf(bqw(J, m, k), u[1 + k], acc);
    y[3 + m] = acc;
  }
#pragma unroll
  for (int n = 0; n < 3; ++n) {
    float acc = x[7 + n];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = fmaf(avq(J, n, j), x[3 + j], acc);
    y[7 + n] = fmaf(bvf(J, n), u[0], acc);
  }
}

// --------------------------------------------------------------------------
// 4x4 Cholesky (lower triangle read, torch.linalg.cholesky semantics)
// --------------------------------------------------------------------------
struct Chol4 {
  float l10, l20, l30, l21, l31, l32;
  float r0, r1, r2, r3;  // reciprocals of the diagonal
};

// 1/sqrt(d): the hardware approximation refined by one Newton-Raphson step
// for the inverse square root, y <- y (3 - d y^2) / 2 (about 1 ulp). Only the
// reciprocals of the diagonal of L enter the solves. Subnormal, zero, negative,
// infinite or NaN d (a failed or degenerate factorisation) take the correctly
// rounded library routine instead.
__device__ __forceinline__ float inv_sqrt(float d) {
  if (!(d >= 1.17549435e-38f && d <= 3.4e38f)) return __frsqrt_rn(d);
  const float y = rsqrtf(d);
  const float h = 0.5f * d * y;
  return fmaf(-h, y * y, 1.5f * y);
}

// chol4's factorisation with the in-range reciprocal square root on every
// pivot and no branch: returns whether every pivot is a positive normal
// number, in which case L holds chol4's bits (and chol4 would return true).
// Otherwise L is meaningless and the caller repeats the factorisation with
// chol4. The straight-line chain lets the scheduler interleave independent
// work with it.
__device__ __forceinline__ bool chol4_fast(const float (&M)[NU][NU], Chol4& L) {
  auto nr = [](float d) {
    const float y = rsqrtf(d);
    const float h = 0.5f * d * y;
    return fmaf(-h, y * y, 1.5f * y);
  };
  auto in_range = [](float d) { return d >= 1.17549435e-38f && d <= 3.4e38f; };
  const float d0 = M[0][0];
  L.r0 = nr(d0);
  L.l10 = M[1][0] * L.r0;
  L.l20 = M[2][0] * L.r0;
  L.l30 = M[3][0] * L.r0;
  const float d1 = M[1][1] - L.l10 * L.l10;
  L.r1 = nr(d1);
  L.l21 = (M[2][1] - L.l20 * L.l10) * L.r1;
  L.l31 = (M[3][1] - L.l30 * L.l10) * L.r1;
  const float d2 = (M[2][2] - L.l20 * L.l20) - L.l21 * L.l21;
  L.r2 = nr(d2);
  L.l32 = ((M[3][2] - L.l30 * L.l20) - L.l31 * L.l21) * L.r2;
  const float d3 = ((M[3][3] - L.l30 * L.l30) - L.l31 * L.l31) - L.l32 * L.l32;
  L.r3 = nr(d3);
  return in_range(d0) & in_range(d1) & in_range(d2) & in_range(d3);
}

__device__ __forceinline__ bool chol4(const float (&M)[NU][NU], Chol4& L) {
  const float d0 = M[0][0];
  L.r0 = inv_sqrt(d0);
  L.l10 = M[1][0] * L.r0;
  L.l20 = M[2][0] * L.r0;
  L.l30 = M[3][0] * L.r0;
  const float d1 = M[1][1] - L.l10 * L.l10;
  L.r1 = inv_sqrt(d1);
  L.l21 = (M[2][1] - L.l20 * L.l10) * L.r1;
  L.l31 = (M[3][1] - L.l30 * L.l10) * L.r1;
  const float d2 = (M[2][2] - L.l20 * L.l20) - L.l21 * L.l21;
  L.r2 = inv_sqrt(d2);
  L.l32 = ((M[3][2] - L.l30 * L.l20) - L.l31 * L.l21) * L.r2;
  const float d3 = ((M[3][3] - L.l30 * L.l30) - L.l31 * L.l31) - L.l32 * L.l32;
  L.r3 = inv_sqrt(d3);
  return (d0 > 0.0f) && (d1 > 0.0f) && (d2 > 0.0f) && (d3 > 0.0f);
}

// x = (L L^T)^-1 b
__device__ __forceinline__ void chol4_solve(const Chol4& L, const float (&b)[NU], float (&x)[NU]) {
  const float y0 = b[0] * L.r0;
  const float y1 = (b[1] - L.l10 * y0) * L.r1;
  const float y2 = ((b[2] - L.l20 * y0) - L.l21 * y1) * L.r2;
  const float y3 = (((b[3] - L.l30 * y0) - L.l31 * y1) - L.l32 * y2) * L.r3;
  x[3] = y3 * L.r3;
  x[2] = (y2 - L.l32 * x[3]) * L.r2;
  x[1] = ((y1 - L.l21 * x[2]) - L.l31 * x[3]) * L.r1;
  x[0] = (((y0 - L.l10 * x[1]) - L.l20 * x[2]) - L.l30 * x[3]) * L.r0;
}

// Fallback inverse for a Q_uu whose Cholesky failed, as _robust_solve's SVD
// branch (DifferentialMPC/controller.py:758-779): M^-1 = V diag(1/S) U^T with
// singular values floored at max(S)/1e12. One-sided Jacobi SVD (Hestenes) on
// the columns of M, a fixed number of sweeps (bounded).
// M and Mi are row-major 4 x 4 arrays (in shared memory for the callers here).
static __device__ __noinline__ void svd_inverse4(const float* M, float* Mi) {
  float W[NU][NU], Vr[NU][NU];
  for (int i = 0; i < NU; ++i)
    for (int j = 0; j < NU; ++j) { W[i][j] = M[i * NU + j]; Vr[i][j] = (i == j) ? 1.0f : 0.0f; }
  for (int sweep = 0; sweep < 12; ++sweep) {
    float off = 0.0f;
    for (int p = 0; p < NU - 1; ++p)
      for (int q = p + 1; q < NU; ++q) {
        float a = 0.0f, b = 0.0f, g = 0.0f;
        for (int i = 0; i < NU; ++i) {
          a = fmaf(W[i][p], W[i][p], a);
          b = fmaf(W[i][q], W[i][q], b);
          g = fmaf(W[i][p], W[i][q], g);
        }
        if (g == 0.0f || fabsf(g) <= 1e-7f * sqrtf(a * b)) continue;
        off = fmaxf(off, fabsf(g) / sqrtf(a * b));
        const float zeta = (b - a) / (2.0f * g);
        const float t = copysignf(1.0f, zeta) / (fabsf(zeta) + sqrtf(1.0f + zeta * zeta));
        const float c = 1.0f / sqrtf(1.0f + t * t);
        const float s = c * t;
        for (int i = 0; i < NU; ++i) {
          const float wp = W[i][p], wq = W[i][q];
          W[i][p] = c * wp - s * wq;
          W[i][q] = s * wp + c * wq;
          const float vp = Vr[i][p], vq = Vr[i][q];
          Vr[i][p] = c * vp - s * vq;
          Vr[i][q] = s * vp + c * vq;
        }
      }
    if (off <= 1e-7f) break;
  }
  float S[NU], smax = 0.0f;
  for (int j = 0; j < NU; ++j) {
    float n2 = 0.0f;
    for (int i = 0; i < NU; ++i) n2 = fmaf(W[i][j], W[i][j], n2);
    S[j] = sqrtf(n2);
    smax = fmaxf(smax, S[j]);
  }
  const float floor_ = smax / 1e12f;
  float R[NU][NU];
  for (int i = 0; i < NU; ++i)
    for (int j = 0; j < NU; ++j) R[i][j] = 0.0f;
  for (int k = 0; k < NU; ++k) {
    if (!(S[k] > 0.0f)) continue;
    const float sr = S[k] > floor_ ? S[k] : floor_;
    const float sc = 1.0f / (S[k] * sr);  // u_k = w_k / S_k, times 1/S_reg
    for (int i = 0; i < NU; ++i)
      for (int j = 0; j < NU; ++j) R[i][j] = fmaf(Vr[i][k] * sc, W[j][k], R[i][j]);
  }
  for (int i = 0; i < NU; ++i)
    for (int j = 0; j < NU; ++j) Mi[i * NU + j] = R[i][j];
}

// --------------------------------------------------------------------------
// Packed FP32 (sm_100): one instruction works on a pair of floats held in a
// 64-bit register pair; each component rounds exactly as fmaf / __fadd_rn /
// __fmul_rn, so a pair of independent scalar operations becomes one
// instruction with the same bits. One exception, measured on B200: a packed
// multiply whose result feeds a packed add can be fused by the code
// generator into one packed FMA (a single rounding), even with -fmad=false
// and even from inline PTX with .rn. The kernels therefore never feed mul2
// into add2; a packed product only starts an FMA chain (as the addend of
// fma2, where no fusion is possible).
// --------------------------------------------------------------------------
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 dup2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }

// --------------------------------------------------------------------------
// cp.async: 16-byte global -> shared copies that complete in the background
// --------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
// 4-byte copy (any 4-byte aligned address), cached in L1 like a plain load.
__device__ __forceinline__ void cp_async_f32(float* smem_dst, const float* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// --------------------------------------------------------------------------
// TMA bulk tensor copies and mbarriers
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait: returns false if the phase did not complete within WAIT_LIMIT polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace ilqr
