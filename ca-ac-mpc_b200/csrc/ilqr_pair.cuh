// ilqr_pair.cuh -- one batch element per half-warp (16 lanes, 2 elements per warp).
//
// The team layout (ilqr_team.cuh) packs six elements into a warp, which
// keeps the instruction count per element low but leaves a small batch with
// too few warps: at B = 2048 it makes 342 warps for 592 schedulers, and each
// element's iterations run as one long serial chain. This layout gives an
// element sixteen lanes: lane i < 10 owns row i of V, lanes 10..13 the four
// control rows, and every phase of a Riccati step spreads over them, so the
// chain per step is several times shorter.
//
// Each output is computed with exactly the operations, in exactly the order,
// of the team kernels, so both layouts give the same bits (for finite
// values: a product with an exact zero coefficient adds a zero here where
// the team formula leaves the term out). To keep every phase one
// instruction stream, each row r in 0..13 of the products A^T Y (Y = V A,
// V B, v) and B^T Y is written in one form,
//     out = base + fmaf(c7, Y[own], sum_s c[s] Y[3 + s]),   s = 0..6,
// the sum accumulated from 0 in index order (pair_coef gives c, c7, own):
//   rows 3..6   column of A at quaternion row r (c7 = 0)
//   row 0       c = 0, c7 = 1, own = 0
//   rows 1, 2   c = 0, c7 = 1, own = r            (position: Y[r])
//   rows 7..9   c[r-3] = 1, c7 = dt, own = r - 7  (velocity: Y[r] + dt Y[p])
//   row 10      c[4..6] = B's thrust column       (Q_uu / q_u row of the thrust)
//   rows 11..13 c[0..3] = B's body-rate column    (Q_uu / q_u rows of the rates)
#pragma once

#include <atomic>
#include <type_traits>

#include "ilqr_device.cuh"
#include "ilqr_kernels.h"
#include "ilqr_team.cuh"

namespace ilqr {

constexpr int HALF = 16;   // lanes per element
constexpr int EPWP = 2;    // elements per warp
// Batches up to this size (and horizons up to PAIR_MAX_T, whose per-step
// tables fit in shared memory) run in the pair layout by default. One wave
// holds 2368 elements (8 CTAs per SM at T = 20); up to 4096 elements (1.73
// waves) the pair layout is still faster than the team layout (B200, T = 20,
// fwd+bwd: B = 2560 10 %, 3072 3 %, 4096 6.5 %), from 5120 it is slower
// (13 % at 5120: a third wave).
constexpr int64_t PAIR_MAX_B = 4096;
constexpr int PAIR_MAX_T = 64;

// Per-element shared-memory area (floats; float4 fields 16-byte aligned).
// Matrices are row-major with rows of 12 floats, so that a float4 load gives
// four columns of a row: two packed pairs.
constexpr int PC0 = 0;       // [2][196] C_t blocks (double buffer; diagonal mode uses block 0)
constexpr int PVA = 392;     // [10][12] rows of V A
constexpr int PVB = 512;     // [10][4]  rows of V B
constexpr int PV = 552;      // [12]     v (v_k at PV + 1 + k: v[3..6], v[7..9] are aligned float4s)
constexpr int PQUU = 564;    // [4][4]   Q_uu rows (reg added once)
constexpr int PQU = 580;     // [4]      q_u
constexpr int PKR = 584;     // [4][12]  rows of K (gain a of every state)
constexpr int PKF = 632;     // [4]      k
constexpr int PQUX = 636;    // [4][12]  rows of Q_ux (Q_xu[c][a] at PQUX + 12 a + c)
constexpr int PS = 684;      // [16]     rowdots s_i = (C_t tau)_i (first-pass objective)
constexpr int PCV = 700;     // [16]     c_t
constexpr int PSV = 716;     // [32]     SVD fallback: Q, its inverse
constexpr int PBASE = 752;   // end of the fixed part of the area
// Per-step tables after the fixed part (floats per step): the nominal record
// (x, u; 16), the Jacobian table (32, below), the gains (ten K columns and k;
// 44) and, in the solve, the cost record (diag C_t, c_t; 32).
constexpr int PREC_F = 16, PJT_F = 32, PKS_F = 44, PCR_F = 32;
// The backward's per-step gradient terms (-dL/dX_t, -dL/dU_t, tight bits; 16).
constexpr int PLX_F = 16;
// Floats per element: the fixed part and `per_t` floats per step, rounded so
// that the two elements' areas start 16 floats apart modulo the 32 banks.
__host__ __device__ __forceinline__ int pair_area(int T, int per_t, int extra = 0) {
  const int n = PBASE + per_t * T + extra;
  return (n + 31) / 32 * 32 + 16;
}

// Jacobian table of one step (32 floats): the fields of Jac and their
// negatives, so that every coefficient of pair_coef is one entry:
//   [0..3] dt h0 h1 h2   [4..7] g0..g3   [8..11] e0..e3   [12..15] bv0 bv1 bv2 1
//   [16..19] 0 -h0 -h1 -h2   [20..23] -g0..-g3   [24..27] -e0..-e3   [28..31] -bv0 -bv1 -bv2 0
__device__ __forceinline__ void jtab_write(float* jt, const Jac& J) {
  float4* q = reinterpret_cast<float4*>(jt);
  q[0] = make_float4(J.dt, J.h0, J.h1, J.h2);
  q[1] = make_float4(J.g0, J.g1, J.g2, J.g3);
  q[2] = make_float4(J.e0, J.e1, J.e2, J.e3);
  q[3] = make_float4(J.bv0, J.bv1, J.bv2, 1.0f);
  q[4] = make_float4(0.0f, -J.h0, -J.h1, -J.h2);
  q[5] = make_float4(-J.g0, -J.g1, -J.g2, -J.g3);
  q[6] = make_float4(-J.e0, -J.e1, -J.e2, -J.e3);
  q[7] = make_float4(-J.bv0, -J.bv1, -J.bv2, 0.0f);
}
__device__ __forceinline__ Jac jtab_read(const float* jt) {
  const float4* q = reinterpret_cast<const float4*>(jt);
  const float4 a = q[0], b = q[1], c = q[2], d = q[3];
  Jac J;
  J.dt = a.x; J.h0 = a.y; J.h1 = a.z; J.h2 = a.w;
  J.g0 = b.x; J.g1 = b.y; J.g2 = b.z; J.g3 = b.w;
  J.e0 = c.x; J.e1 = c.y; J.e2 = c.z; J.e3 = c.w;
  J.bv0 = d.x; J.bv1 = d.y; J.bv2 = d.z;
  return J;
}

// Coefficients of row r (0..13) in the form of the header comment.
// (Evaluated once per kernel on a probe Jacobian whose fields are distinct
// small integers, to find which Jacobian-table entry each coefficient is;
// pair_coef_offsets.)
__device__ __forceinline__ void pair_coef(const Jac& J, int r, float (&c)[7], float& c7, int& own) {
  const float z = 0.0f;
  float cc[8];
  coef_a(J, (r >= 3 && r <= 6) ? r - 3 : 4, cc);  // rows 3..6; m = 4 gives zeros and cc[7] = 1
#pragma unroll
  for (int s = 0; s < 7; ++s) c[s] = (r >= 3 && r <= 6) ? cc[s] : z;
  c7 = (r <= 6) ? cc[7] : z;  // rows 0..2: 1; rows 3..6: 0
  own = r < 3 ? r : (r <= 6 ? r : (r < NX ? r - 7 : 0));
  if (r >= 7 && r < NX) {
#pragma unroll
    for (int s = 4; s < 7; ++s) c[s] = (s == r - 3) ? 1.0f : z;
    c7 = J.dt;
  }
  if (r == NX) {
    c[4] = J.bv0;
    c[5] = J.bv1;
    c[6] = J.bv2;
  }
  if (r > NX) {
    const int kk = r - NX - 1;
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) c[mm] = kk == 0 ? bqw(J, mm, 0) : (kk == 1 ? bqw(J, mm, 1) : bqw(J, mm, 2));
  }
}

// Jacobian-table offsets of row r's coefficients c[0..6] and c7 (5 bits
// each, packed), found by evaluating pair_coef on a probe whose fields are
// the codes 2..16: a coefficient 0 is entry 16, 1 is entry 15, field k is
// entry k and its negative entry 16 + k.
__device__ __forceinline__ uint64_t pair_coef_offsets(int r, int& own) {
  Jac P;
  P.dt = 2.0f; P.h0 = 3.0f; P.h1 = 4.0f; P.h2 = 5.0f;
  P.g0 = 6.0f; P.g1 = 7.0f; P.g2 = 8.0f; P.g3 = 9.0f;
  P.e0 = 10.0f; P.e1 = 11.0f; P.e2 = 12.0f; P.e3 = 13.0f;
  P.bv0 = 14.0f; P.bv1 = 15.0f; P.bv2 = 16.0f;
  float c[7], c7;
  pair_coef(P, r, c, c7, own);
  auto off = [](float v) -> uint64_t {
    const int k = (int)fabsf(v) - 2;
    return v == 0.0f ? 16u : (v == 1.0f ? 15u : (v > 0.0f ? (uint64_t)k : (uint64_t)(16 + k)));
  };
  uint64_t o = 0;
#pragma unroll
  for (int s = 0; s < 7; ++s) o |= off(c[s]) << (5 * s);
  o |= off(c7) << 35;
  return o;
}

// Row coefficients of one step from its Jacobian table.
__device__ __forceinline__ void pair_coef_load(const float* jt, uint64_t offs, float (&c)[7], float& c7) {
#pragma unroll
  for (int s = 0; s < 7; ++s) c[s] = jt[(offs >> (5 * s)) & 31u];
  c7 = jt[(offs >> 35) & 31u];
}

// One Riccati step for an element's half-warp; the same recursion and
// operation order as team_riccati (ilqr_team.cuh), forward or masked.
// c, c7, own: the coefficients of this lane's row (pair_coef, through the
// step's Jacobian table; lanes 14, 15 carry row 13's).
// Lane i < 10: Vr, vr = row i of V and v_i (in V_{t+1}, out V_t). lx_fn():
// lane i < 10 the gradient term of row i, lane 10 + a that of control a;
// called first, so that its arithmetic overlaps the rows of V A. Ce: the
// element's C_t block in shared memory. sh: the element's area. On return
// lane i < 10 holds column i of K in Kr (the four gains of state i), lane 10
// holds k. Every lane returns whether the Cholesky succeeded (the same in all
// lanes of the half). Ends with a warp sync: C_t and the area are free.
template <bool MASKED, class LxFn>
__device__ __forceinline__ bool pair_riccati(float (&Vr)[NX], float& vr, const Jac& J, const float (&c)[7], float c7,
                                             int own, const float* __restrict__ Ce, LxFn&& lx_fn, float reg,
                                             uint32_t tight, int i, bool live, float* __restrict__ sh,
                                             float (&Kr)[NU]) {
  const float lx = lx_fn();
  // ---- rows of V A (as columns of VAT), V B and v ----------------------------
  // (Lanes 10..15 run every phase on a stand-in row, which keeps the warp in
  // one instruction stream; only the lanes of real rows store.)
  {
    float va[NX], vb[NU];
    row_VA_VB(J, Vr, va, vb);
    if (i < NX) {
      float* row = sh + PVA + 12 * i;
      *reinterpret_cast<float4*>(row) = make_float4(va[0], va[1], va[2], va[3]);
      *reinterpret_cast<float4*>(row + 4) = make_float4(va[4], va[5], va[6], va[7]);
      *reinterpret_cast<float2*>(row + 8) = make_float2(va[8], va[9]);
      *reinterpret_cast<float4*>(sh + PVB + 4 * i) = make_float4(vb[0], vb[1], vb[2], vb[3]);
      sh[PV + 1 + i] = vr;
    }
  }
  __syncwarp();

  // ---- Q_xu rows and q_x (lanes 0..9), Q_uu rows and q_u (lanes 10..13) -------
  const int r = i < NT ? i : NT - 1;
  // the row's coefficients as packed pairs (the same value in both halves)
  float2 c2[7];
#pragma unroll
  for (int s = 0; s < 7; ++s) c2[s] = dup2(c[s]);
  const float2 c72 = dup2(c7);
  float Qr[NU], qr;
  {
    float2 acc01 = make_float2(0.0f, 0.0f), acc23 = make_float2(0.0f, 0.0f);
    float accv = 0.0f;
    const float4 v36 = *reinterpret_cast<const float4*>(sh + PV + 4);
    const float4 v79 = *reinterpret_cast<const float4*>(sh + PV + 8);
    const float vs[7] = {v36.x, v36.y, v36.z, v36.w, v79.x, v79.y, v79.z};
#pragma unroll
    for (int s = 0; s < 7; ++s) {
      const float* y = sh + PVB + 4 * (3 + s);
      acc01 = fma2(c2[s], ld2(y), acc01);
      acc23 = fma2(c2[s], ld2(y + 2), acc23);
      accv = fmaf(c[s], vs[s], accv);
    }
    const float* o = sh + PVB + 4 * own;
    const float* Cr = Ce + r * NT + NX;
    float2 q01 = add2(ld2(Cr), fma2(c72, ld2(o), acc01));
    float2 q23 = add2(ld2(Cr + 2), fma2(c72, ld2(o + 2), acc23));
    if (r >= NX) {
      q01 = add2(q01, make_float2(r - NX == 0 ? reg : 0.0f, r - NX == 1 ? reg : 0.0f));
      q23 = add2(q23, make_float2(r - NX == 2 ? reg : 0.0f, r - NX == 3 ? reg : 0.0f));
    }
    Qr[0] = q01.x; Qr[1] = q01.y; Qr[2] = q23.x; Qr[3] = q23.y;
    qr = lx + fmaf(c7, sh[PV + 1 + own], accv);
  }
  if (i >= NX && i < NT) {
    *reinterpret_cast<float4*>(sh + PQUU + 4 * (i - NX)) = make_float4(Qr[0], Qr[1], Qr[2], Qr[3]);
    sh[PQU + i - NX] = qr;
  }
  if (i < NX) {
#pragma unroll
    for (int a = 0; a < NU; ++a) sh[PQUX + 12 * a + i] = Qr[a];
  }
  __syncwarp();

  // ---- gains: every lane factors Q_uu, lane i < 10 solves column i of K,
  // lane 10 solves k ----------------------------------------------------------
  float Quu[NU][NU], qu[NU];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    const float4 q4 = *reinterpret_cast<const float4*>(sh + PQUU + 4 * a);
    Quu[a][0] = q4.x; Quu[a][1] = q4.y; Quu[a][2] = q4.z; Quu[a][3] = q4.w;
  }
  {
    const float4 q4 = *reinterpret_cast<const float4*>(sh + PQU);
    qu[0] = q4.x; qu[1] = q4.y; qu[2] = q4.z; qu[3] = q4.w;
  }
  // Q_xx[i][cc] = C_t[i][cc] + (A^T (V A))[i][cc] for the value update, as
  // packed pairs of columns: independent of the gains, so formed here, where
  // its products fill the latency of the factorisation's serial chain.
  const float* Crow = Ce + (i < NX ? i : NX - 1) * NT;
  float2 qxx[NX / 2];
  {
#pragma unroll
    for (int hh = 0; hh < NX / 2; ++hh) qxx[hh] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int s = 0; s < 7; ++s) {
      const float* y = sh + PVA + 12 * (3 + s);
#pragma unroll
      for (int hh = 0; hh < NX / 2; ++hh) qxx[hh] = fma2(c2[s], ld2(y + 2 * hh), qxx[hh]);
    }
#pragma unroll
    for (int hh = 0; hh < NX / 2; ++hh) {
      const int cc = 2 * hh;
      qxx[hh] = add2(ld2(Crow + cc), fma2(c72, ld2(sh + PVA + 12 * own + cc), qxx[hh]));
    }
  }
  // The common case runs straight through: the factorisation with in-range
  // pivots and the triangular solves. A warp with a pivot outside the normal
  // range (Q_uu not positive definite, or degenerate) repeats them for those
  // lanes through chol4 and, where that fails, the SVD inverse.
  Chol4 L;
  float Qs[NU][NU];
#pragma unroll
  for (int a = 0; a < NU; ++a)
#pragma unroll
    for (int b = 0; b < NU; ++b) {
      if (MASKED) {
        const bool ta = (tight >> a) & 1u, tb = (tight >> b) & 1u;
        float val = (ta || tb) ? 0.0f : Quu[a][b];
        if (a == b && ta) val = val + 1.0f;
        Qs[a][b] = val + (a == b ? 1e-8f * reg : 0.0f);
      } else {
        Qs[a][b] = Quu[a][b] + (a == b ? reg : 0.0f);
      }
    }
  const bool inr = chol4_fast(Qs, L);
  auto msk = [&](int a, float v) { return (MASKED && ((tight >> a) & 1u)) ? 0.0f : v; };
  float rhs[NU], sol[NU];
#pragma unroll
  for (int a = 0; a < NU; ++a) rhs[a] = msk(a, i < NX ? Qr[a] : qu[a]);
  chol4_solve(L, rhs, sol);
  bool ok = true;
  if (__any_sync(FULL, !inr)) {
    float* sv = sh + PSV;
    if (!inr) {
      // A half without an element never takes the SVD path.
      ok = chol4(Qs, L) || !live;
      if (!ok) {
        // every lane of the half forms the same inverse; identical writes
#pragma unroll
        for (int a = 0; a < NU; ++a)
#pragma unroll
          for (int b = 0; b < NU; ++b) sv[a * NU + b] = Qs[a][b];
        svd_inverse4(sv, sv + NU * NU);
      }
    }
    if (__any_sync(FULL, !ok)) __syncwarp();  // every fallback inverse of the warp is written
    if (!inr) {
      if (ok) {
        chol4_solve(L, rhs, sol);
      } else {
        const float* Mi = sv + NU * NU;
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          float acc = Mi[a * NU] * rhs[0];
#pragma unroll
          for (int b = 1; b < NU; ++b) acc = fmaf(Mi[a * NU + b], rhs[b], acc);
          sol[a] = acc;
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < NU; ++a) Kr[a] = -sol[a];
  if (i < NX) {
#pragma unroll
    for (int a = 0; a < NU; ++a) sh[PKR + 12 * a + i] = Kr[a];
  }
  if (i == NX) *reinterpret_cast<float4*>(sh + PKF) = make_float4(Kr[0], Kr[1], Kr[2], Kr[3]);
  // W_r = K_r^T Q_uu + Q_xu[r] (team_riccati's wrow)
  float Wr[NU];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    float acc = Kr[0] * Quu[0][a];
#pragma unroll
    for (int b = 1; b < NU; ++b) acc = fmaf(Kr[b], Quu[b][a], acc);
    Wr[a] = acc + Qr[a];
  }
  __syncwarp();  // K columns and k of the element are in the area

  // ---- value update for row i ---------------------------------------------
  float k[NU];
  {
    const float4 k4 = *reinterpret_cast<const float4*>(sh + PKF);
    k[0] = k4.x; k[1] = k4.y; k[2] = k4.z; k[3] = k4.w;
  }
  {
    if (MASKED) {
      float w[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        float acc = Quu[a][0] * k[0];
#pragma unroll
        for (int b = 1; b < NU; ++b) acc = fmaf(Quu[a][b], k[b], acc);
        w[a] = acc + qu[a];
      }
      float t2 = Kr[0] * w[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t2 = fmaf(Kr[a], w[a], t2);
      float t3 = Qr[0] * k[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t3 = fmaf(Qr[a], k[a], t3);
      vr = (qr + t2) + t3;
    } else {
      float t1 = Wr[0] * k[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t1 = fmaf(Wr[a], k[a], t1);
      float t2 = Kr[0] * qu[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t2 = fmaf(Kr[a], qu[a], t2);
      vr = (qr + t1) + t2;
    }
    // V[i][cc] = (Q_xx[i][cc] + W_i K_cc) + K_i Q_xu[cc] (Q_xx formed before
    // the factorisation); packed pairs of columns (cc, cc + 1), every sum in
    // the order of the scalar formula.
    float2 w2[NU], kr2[NU];
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      w2[a] = dup2(Wr[a]);
      kr2[a] = dup2(Kr[a]);
    }
#pragma unroll
    for (int hh = 0; hh < NX / 2; ++hh) {
      const int cc = 2 * hh;
      float2 t1 = mul2(w2[0], ld2(sh + PKR + cc));
#pragma unroll
      for (int a = 1; a < NU; ++a) t1 = fma2(w2[a], ld2(sh + PKR + 12 * a + cc), t1);
      float2 t2 = mul2(kr2[0], ld2(sh + PQUX + cc));
#pragma unroll
      for (int a = 1; a < NU; ++a) t2 = fma2(kr2[a], ld2(sh + PQUX + 12 * a + cc), t2);
      const float2 v = add2(add2(qxx[hh], t1), t2);
      Vr[cc] = v.x;
      Vr[cc + 1] = v.y;
    }
  }
  __syncwarp();  // C_t and the area are no longer read
  return ok;
}

// Raise a kernel's dynamic shared-memory limit to `bytes` (above the default
// 48 KB the launch needs it; harmless below).
// Set once per kernel and size (a later, larger request sets it again), so
// that launches recorded into a CUDA graph call no attribute setter.
template <auto Kernel>
inline cudaError_t allow_smem(size_t bytes) {
  static std::atomic<size_t> granted{0};  // one per kernel
  if (bytes <= granted.load()) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) granted.store(bytes);
  return e;
}

// Sum of x over lanes base .. base + 4 in that order (team_sum's order).
__device__ __forceinline__ float pair_sum5(float x, int base) {
  float s = __shfl_sync(FULL, x, base);
#pragma unroll
  for (int j = 1; j < TEAM; ++j) s += __shfl_sync(FULL, x, base + j);
  return s;
}

// cp.async stream of one element's C_t blocks (16 lanes, 49 copies of 16
// bytes per block) through two buffers (buf) or, with a third buffer (buf3),
// three: issue(t) copies block t into buffer t mod depth; each lane commits
// one group per issue. With three buffers a pass can keep two blocks in
// flight while it works on a third.
struct PairCPipe {
  const float* Cb;   // C block of (element, t) at Cb + t * tstride * CBLK
  int64_t tstride;
  float* buf;        // the element's area + PC0 (two blocks)
  int i;
  float* buf3 = nullptr;  // a third block's buffer, or none
  __device__ __forceinline__ float* block(int t) const {
    if (buf3 != nullptr) {
      const int r = t % 3;
      return r == 2 ? buf3 : buf + r * CBLK;
    }
    return buf + (t & 1) * CBLK;
  }
  __device__ __forceinline__ void issue(int t) {
    const float* src = Cb + (int64_t)t * tstride * CBLK;
    float* dst = block(t);
    for (int q = i; q < CBLK / 4; q += HALF) cp_async16(dst + 4 * q, src + 4 * q);
    cp_async_commit();
  }
};

}  // namespace ilqr
