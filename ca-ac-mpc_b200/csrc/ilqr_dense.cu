// ilqr_dense.cu -- fused iLQR solve and implicit-diff backward for the
// 13-state rotor-thrust quadrotor (ilqr_rotor13.cuh).
//
// The same algorithm as ilqr_solve.cu / ilqr_backward.cu (DiffMPC semantics:
// DifferentialMPC/controller.py:303-533 solve loop, Riccati and grid line
// search, :997-1003 tight mask, :68-133 and :1006-1131 implicit-diff backward),
// for a model whose Jacobians are dense enough that a row-per-lane layout
// pays: one batch element per group of 16 lanes, two elements per warp.
//
// Riccati step (lanes 0..12 own the state rows i, lanes 0..3 also the control
// rows, all 16 lanes the 4 x 4 Q_uu entries), matrices in shared memory:
//   J   lane i writes row i of A_t, B_t (from the nominal x_t, u_t)
//   P1  (V B)_i., (A^T V)_i. = sum_k A_ki V_k., q_x,i ; q_u (lanes 0..3)
//   P2  Q_xx,i. = C_xx,i. + (A^T V)_i. A ; Q_xu,i. = C_xu,i. + A_.i^T (V B)
//       Q_uu,ab = C_uu,ab + B_.a^T (V B)_.b + reg [a = b]   (one entry per lane)
//   P3  K_.i = -(Q_uu + reg I)^-1 Q_xu,i.^T by a Cholesky every lane repeats
//       (SVD inverse when it fails); k by lane 13; M = Q_uu K + Q_ux
//   P4  V_i. = Q_xx,i. + K_.i^T M + Q_xu,i. K ; v_i likewise
// with a warp barrier after each. The line search runs one step size per lane
// (lane j rolls out candidate j over the horizon), so the n_alpha candidates
// of an element run side by side; each candidate trajectory is kept in its
// own workspace slot and the accepted one becomes the nominal.
#include <cstdint>

#include "ilqr_b200.h"
#include "ilqr_device.cuh"
#include "ilqr_kernels.h"
#include "ilqr_rotor13.cuh"

namespace ilqr {
namespace r13 {

namespace {

constexpr int GL = 16;             // lanes per element
constexpr int EPW = 2;             // elements per warp
constexpr int WPC = 4;             // warps per CTA (backward)
constexpr int EPC = EPW * WPC;     // elements per CTA (backward)
constexpr int THREADS = WPC * 32;  // threads per CTA (backward)
// The solve launches one-warp CTAs: its warps share nothing, and its
// elements run 1 to max_iter iterations (at B = 16384, T = 20, 5 iterations,
// 63 % stop after one), so a CTA should free its registers as soon as its
// own two elements are done, not when the slowest of eight is.
constexpr int S_WPC = 1;
constexpr int S_EPC = EPW * S_WPC;
constexpr int S_THREADS = S_WPC * 32;
constexpr int REC = 20;            // floats per trajectory record: x[13], u[4], 3 pad
constexpr int SM_COUNT = 148;      // B200 SMs (the launch's one-wave test)

// Shared memory of one element (floats). The block size is an odd multiple
// of 16 floats, so the two elements of a warp use opposite halves of the
// banks for the same offsets.
// V, A_t, K_t and M have rows of LDM = 14 floats (13 used), so that two
// adjacent columns of a row are one 8-byte load: a packed pair.
constexpr int LDM = 14;
constexpr int S_V = 0;       // V [13][14]
constexpr int S_A = 184;     // A_t [13][14]
constexpr int S_B = 368;     // B_t [13][4]
constexpr int S_VB = 420;    // V B [13][4]
constexpr int S_K = 472;     // K_t [4][14]
constexpr int S_M = 528;     // Q_uu K + Q_ux [4][14]
constexpr int S_VV = 584;    // v [13]
constexpr int S_Z = 600;     // nominal x_t, u_t [20]
constexpr int S_QUU = 620;   // Q_uu [4][4] (regularised once)
constexpr int S_QU = 636;    // q_u [4]
constexpr int S_KF = 640;    // k_t [4]
constexpr int S_MK = 644;    // Q_uu k + q_u [4]
constexpr int S_SVD = 648;   // SVD fallback: matrix [16], inverse [16]
constexpr int S_TAU = 680;   // per-lane tau scratch of the rollouts [16][17]
constexpr int S_LS2 = 952;   // second rollout staging buffer (the first is at 0)
constexpr int S_ELEM = 1360; // floats per element in the solve (85 x 16)
constexpr int S_STG = 944;   // backward: two buffers staging a step's inputs
constexpr int S_ELEM_BWD = 1616;  // floats per element in the backward (101 x 16)
// One staged backward step (floats, relative to a buffer): C_t (in the tangent
// sweep the K_t columns and k_t as 14 float4), the tight mask (4 bytes), x_t and
// u_t, dL/dX_t, dL/dU_t.
constexpr int R_C = 0;
constexpr int R_TM = 289;
constexpr int R_REC = 292;
constexpr int R_GX = 312;
constexpr int R_GU = 325;
constexpr int R_SIZE = 332;
// Outside the Riccati pass the first 404 floats stage one step of a rollout:
// C_t (289), c_t (17), x_ref_t (13), u_ref_t (4), U_init_t (4), then the
// nominal record (20) and the K_t columns and k_t (56) as float4s.
constexpr int L_C = 0;
constexpr int L_CV = 289;
constexpr int L_XR = 306;
constexpr int L_UR = 319;
constexpr int L_U0 = 323;
constexpr int L_NSC = 327;   // staged scalars
constexpr int L_F4 = 328;    // float4 area: record (5), K columns and k (14)
constexpr int L_NF4 = 19;
constexpr int L_PF = 21;     // scalar prefetch slots per lane (16 x 21 >= 327)

// 4-byte global -> shared copy completing in the background (cp.async groups
// as cp_async16's).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ float clampn(float v, float lo, float hi) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(v), "f"(lo));
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(r), "f"(hi));
  return r;
}

__device__ __forceinline__ float group_sum(float v, unsigned mask) {
#pragma unroll
  for (int o = GL / 2; o > 0; o >>= 1) v += __shfl_xor_sync(mask, v, o);
  return v;
}

// Workspace of one element (floats, element-major):
//   slots  [n_slot][T+1][REC]   trajectory records
//   K cols [T][13] float4        column j of K_t (the four gains of state j)
//   k      [T] float4
struct Ws {
  float* base;
  int T;
  int n_slot;
  __device__ float4* rec(int slot, int t) const {
    return reinterpret_cast<float4*>(base + ((int64_t)slot * (T + 1) + t) * REC);
  }
  __device__ float4* kcol(int t, int j) const {
    return reinterpret_cast<float4*>(base + (int64_t)n_slot * (T + 1) * REC) + (int64_t)t * (NX + 1) + j;
  }
  __device__ float4* kff(int t) const { return kcol(t, NX); }
};

__device__ __forceinline__ void load_rec(const float4* r, float* x, float* u) {
  const float4 a = r[0], b = r[1], c = r[2], d = r[3], e = r[4];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  x[8] = c.x; x[9] = c.y; x[10] = c.z; x[11] = c.w;
  x[12] = d.x; u[0] = d.y; u[1] = d.z; u[2] = d.w;
  u[3] = e.x;
}

__device__ __forceinline__ void store_rec(float4* r, const float* x, const float* u) {
  r[0] = make_float4(x[0], x[1], x[2], x[3]);
  r[1] = make_float4(x[4], x[5], x[6], x[7]);
  r[2] = make_float4(x[8], x[9], x[10], x[11]);
  r[3] = make_float4(x[12], u[0], u[1], u[2]);
  r[4] = make_float4(u[3], 0.0f, 0.0f, 0.0f);
}

// The rows r, r + n, r + 2n, ... of tau^T C tau (C_t staged), with tau_i read
// from this lane's scratch ts (the row index is not a compile-time constant).
__device__ __forceinline__ float step_quad_rows(const float* st, const float* tau, const float* ts, int r, int n) {
  float q = 0.0f;
  for (int i = r; i < NT; i += n) {
    const float* row = st + L_C + i * NT;
    float v = row[0] * tau[0];
#pragma unroll
    for (int j = 1; j < NT; ++j) v = fmaf(row[j], tau[j], v);
    q = fmaf(ts[i], v, q);
  }
  return q;
}

// Lanes per line-search candidate when n candidates share an element's 16 lanes.
__device__ __forceinline__ int lanes_per_candidate(int n) { return n <= 4 ? 4 : (n <= 5 ? 3 : 2); }

// Terminal cost 1/2 tN^T C_f tN + c_f^T tN, tN = [x_T - x_ref_T; 0].
__device__ __forceinline__ float terminal_cost(const float* __restrict__ Cf, const float* __restrict__ cf,
                                               const float* tn) {
  if (Cf == nullptr) return 0.0f;
  float q = 0.0f, l = 0.0f;
#pragma unroll
  for (int i = 0; i < NX; ++i) {
    const float* row = Cf + i * NT;
    float r = __ldg(row) * tn[0];
#pragma unroll
    for (int j = 1; j < NX; ++j) r = fmaf(__ldg(row + j), tn[j], r);
    q = fmaf(tn[i], r, q);
    if (cf != nullptr) l = fmaf(__ldg(cf + i), tn[i], l);
  }
  return 0.5f * q + l;
}

// x = M^-1 b for one 4 x 4 system by Gaussian elimination with partial
// pivoting (M and b are copies). Returns the smallest and largest pivot
// magnitudes: a ratio below 1e-12 (or a non-finite pivot) marks M as
// singular to working precision.
__device__ __forceinline__ void lu_solve4(const float (&Min)[NU][NU], const float (&bin)[NU], float (&x)[NU],
                                          float& pmin, float& pmax) {
  float M[NU][NU], b[NU];
#pragma unroll
  for (int i = 0; i < NU; ++i) {
#pragma unroll
    for (int j = 0; j < NU; ++j) M[i][j] = Min[i][j];
    b[i] = bin[i];
  }
  pmin = 3.4e38f;
  pmax = 0.0f;
#pragma unroll
  for (int k = 0; k < NU; ++k) {
    int r = k;
    float best = fabsf(M[k][k]);
#pragma unroll
    for (int i = k + 1; i < NU; ++i) {
      const float v = fabsf(M[i][k]);
      if (v > best) {
        best = v;
        r = i;
      }
    }
#pragma unroll
    for (int i = k + 1; i < NU; ++i) {
      if (i == r) {
#pragma unroll
        for (int j = 0; j < NU; ++j) {
          const float t = M[k][j];
          M[k][j] = M[i][j];
          M[i][j] = t;
        }
        const float t = b[k];
        b[k] = b[i];
        b[i] = t;
      }
    }
    const float piv = M[k][k];
    pmin = fminf(pmin, fabsf(piv));
    pmax = fmaxf(pmax, fabsf(piv));
#pragma unroll
    for (int i = k + 1; i < NU; ++i) {
      const float f = M[i][k] / piv;
#pragma unroll
      for (int j = k + 1; j < NU; ++j) M[i][j] = M[i][j] - f * M[k][j];
      b[i] = b[i] - f * b[k];
    }
  }
#pragma unroll
  for (int i = NU - 1; i >= 0; --i) {
    float s = b[i];
#pragma unroll
    for (int j = i + 1; j < NU; ++j) s = s - M[i][j] * x[j];
    x[i] = s / M[i][i];
  }
}

// Structural nonzeros of the rotor model's A_t by column (rows k with A_kj
// possibly nonzero; ilqr_rotor13.cuh): p columns only their diagonal, quaternion
// columns the quaternion and velocity rows, velocity columns the position row
// and the diagonal, rate columns the quaternion and rate rows. B_t is zero in
// rows 0..6. Products over these sets skip exact zeros only, so they round as
// the dense products (for finite values).
__host__ __device__ constexpr int a_col_nnz(int j) { return j < 3 ? 1 : (j < 7 ? 7 : (j < 10 ? 2 : 7)); }
__host__ __device__ constexpr int a_col_row(int j, int m) {
  return j < 3 ? j
               : (j < 7 ? 3 + m : (j < 10 ? (m == 0 ? j - 7 : j) : (m < 4 ? 3 + m : 6 + m)));
}
constexpr int B_ROW0 = 7;  // first row of B_t that can be nonzero

// Inputs of one Riccati step that differ between the solve and the backward.
struct StepIn {
  float lx;       // l_x,i (state-row lanes)
  float lu;       // l_u,a for a = lane (lanes 0..3)
  float cxx[NX];  // C_xx,i.
  float cxu[NU];  // C_xu,i.
  float cuu;      // C_uu,ab for (a, b) = (lane / 4, lane % 4)
};

// One step of the Riccati recursion for the element of this lane's group.
// MASKED selects the implicit-diff form (_zero_constrained_lqr,
// controller.py:1070-1110): tight rows/columns of Q_uu replaced by the
// identity plus a (1e-8 reg) I ridge for the gain solve, tight rows of Q_ux
// and entries of q_u zeroed; otherwise the forward form (backward_lqr,
// controller.py:697-723) solves with Q_uu + reg I (reg a second time).
// V and v are updated with the unmasked Q_uu (once regularised), Q_ux, q_u.
// Returns true if the Cholesky failed and the SVD inverse was used.
template <bool MASKED>
__device__ __forceinline__ bool riccati_step(float* sm, int g, bool rowx, bool live, unsigned wmask, const StepIn& in,
                                             float reg, const bool* tight, float (&Vr)[NX], float& vi, float (&Kc)[NU],
                                             float (&kf)[NU]) {
  // ---- P1 ---------------------------------------------------------------
  float acol[NX];
#pragma unroll
  for (int k = 0; k < NX; ++k) acol[k] = rowx ? sm[S_A + k * LDM + g] : 0.0f;
  float w[NX];
  float qx = 0.0f;
  // the column of A as packed pairs (the same value in both halves)
  float2 ac2[NX];
#pragma unroll
  for (int k = 0; k < NX; ++k) ac2[k] = dup2(acol[k]);
  if (rowx) {
    {
      // (V B)_g. over the two column pairs of B
      float2 vb[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float2 s = mul2(dup2(Vr[B_ROW0]), ld2(sm + S_B + B_ROW0 * NU + 2 * h));
#pragma unroll
        for (int k = B_ROW0 + 1; k < NX; ++k) s = fma2(dup2(Vr[k]), ld2(sm + S_B + k * NU + 2 * h), s);
        vb[h] = s;
      }
      *reinterpret_cast<float4*>(sm + S_VB + g * NU) = make_float4(vb[0].x, vb[0].y, vb[1].x, vb[1].y);
    }
    // w = (A^T V)_g. by column pairs (j, j + 1), column 12 alone
#pragma unroll
    for (int j = 0; j < NX - 1; j += 2) {
      float2 s = mul2(ac2[0], ld2(sm + S_V + j));
#pragma unroll
      for (int k = 1; k < NX; ++k) s = fma2(ac2[k], ld2(sm + S_V + k * LDM + j), s);
      w[j] = s.x;
      w[j + 1] = s.y;
    }
    {
      float s = acol[0] * sm[S_V + NX - 1];
#pragma unroll
      for (int k = 1; k < NX; ++k) s = fmaf(acol[k], sm[S_V + k * LDM + NX - 1], s);
      w[NX - 1] = s;
    }
    float s = acol[0] * sm[S_VV];
#pragma unroll
    for (int k = 1; k < NX; ++k) s = fmaf(acol[k], sm[S_VV + k], s);
    qx = in.lx + s;
  }
  if (g < NU) {
    float s = sm[S_B + B_ROW0 * NU + g] * sm[S_VV + B_ROW0];
#pragma unroll
    for (int k = B_ROW0 + 1; k < NX; ++k) s = fmaf(sm[S_B + k * NU + g], sm[S_VV + k], s);
    sm[S_QU + g] = in.lu + s;
  }
  __syncwarp(wmask);
  // ---- P2 ---------------------------------------------------------------
  float qxx[NX], qxu[NU];
  if (rowx) {
#pragma unroll
    for (int j = 0; j < NX; ++j) {
      const int k0 = a_col_row(j, 0);
      float s = w[k0] * sm[S_A + k0 * LDM + j];
#pragma unroll
      for (int m = 1; m < 7; ++m) {
        if (m < a_col_nnz(j)) {
          const int k = a_col_row(j, m);
          s = fmaf(w[k], sm[S_A + k * LDM + j], s);
        }
      }
      qxx[j] = in.cxx[j] + s;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float2 s = mul2(ac2[0], ld2(sm + S_VB + 2 * h));
#pragma unroll
      for (int k = 1; k < NX; ++k) s = fma2(ac2[k], ld2(sm + S_VB + k * NU + 2 * h), s);
      qxu[2 * h] = in.cxu[2 * h] + s.x;
      qxu[2 * h + 1] = in.cxu[2 * h + 1] + s.y;
    }
  }
  {
    const int a = g >> 2, b = g & 3;
    float s = sm[S_B + B_ROW0 * NU + a] * sm[S_VB + B_ROW0 * NU + b];
#pragma unroll
    for (int k = B_ROW0 + 1; k < NX; ++k) s = fmaf(sm[S_B + k * NU + a], sm[S_VB + k * NU + b], s);
    float q = in.cuu + s;
    if (a == b) q = q + reg;
    sm[S_QUU + g] = q;
  }
  __syncwarp(wmask);
  // ---- P3: gains ----------------------------------------------------------
  float Q[NU][NU], qu[NU];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
#pragma unroll
    for (int b = 0; b < NU; ++b) Q[a][b] = sm[S_QUU + a * NU + b];
    qu[a] = sm[S_QU + a];
  }
  bool msk[NU] = {false, false, false, false};
  if (MASKED) {
#pragma unroll
    for (int a = 0; a < NU; ++a) msk[a] = tight[a];
  }
  float G[NU][NU];  // the matrix the gains are solved with
#pragma unroll
  for (int a = 0; a < NU; ++a)
#pragma unroll
    for (int b = 0; b < NU; ++b) {
      if (MASKED) {
        float v = (msk[a] || msk[b]) ? 0.0f : Q[a][b];
        if (a == b && msk[a]) v = v + 1.0f;
        if (a == b) v = v + 1e-8f * reg;
        G[a][b] = v;
      } else {
        G[a][b] = (a == b) ? Q[a][b] + reg : Q[a][b];
      }
    }
  float rhs[NU];
  if (g < NX) {
#pragma unroll
    for (int a = 0; a < NU; ++a) rhs[a] = (MASKED && msk[a]) ? 0.0f : qxu[a];
  } else {
#pragma unroll
    for (int a = 0; a < NU; ++a) rhs[a] = (MASKED && msk[a]) ? 0.0f : qu[a];
  }
  Chol4 L;
  const bool ok = chol4(G, L);
  float sol[NU];
  const bool fb = !ok && live;
  // A failed Cholesky falls back to the inverse: the reference takes an SVD
  // pseudo-inverse with singular values floored at max / 1e12 in the forward
  // Riccati (controller.py:758-779) and an LU solve in the masked one
  // (controller.py:1089-1092). Both equal the LU solve unless the matrix is
  // singular to that ratio; only then is the SVD inverse formed.
  bool sing = false;
  if (ok) {
    chol4_solve(L, rhs, sol);
  } else {
    float pmin, pmax;
    lu_solve4(G, rhs, sol, pmin, pmax);
    sing = !MASKED && !(pmin > 1e-12f * pmax);
  }
  const bool need_svd = sing && live;
  if (__any_sync(wmask, need_svd)) {
    float* M = sm + S_SVD;
    if (need_svd && g == 0) {
#pragma unroll
      for (int a = 0; a < NU; ++a)
#pragma unroll
        for (int b = 0; b < NU; ++b) M[a * NU + b] = G[a][b];
      svd_inverse4(M, M + 16);
    }
    __syncwarp(wmask);
    if (need_svd) {
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        float s = M[16 + a * NU] * rhs[0];
#pragma unroll
        for (int b = 1; b < NU; ++b) s = fmaf(M[16 + a * NU + b], rhs[b], s);
        sol[a] = s;
      }
    }
    __syncwarp(wmask);
  }
#pragma unroll
  for (int a = 0; a < NU; ++a) sol[a] = -sol[a];
  if (rowx) {
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      Kc[a] = sol[a];
      sm[S_K + a * LDM + g] = sol[a];
    }
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      float s = Q[a][0] * sol[0];
#pragma unroll
      for (int b = 1; b < NU; ++b) s = fmaf(Q[a][b], sol[b], s);
      sm[S_M + a * LDM + g] = s + qxu[a];
    }
  } else if (g == NX) {
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      kf[a] = sol[a];
      sm[S_KF + a] = sol[a];
    }
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      float s = Q[a][0] * sol[0];
#pragma unroll
      for (int b = 1; b < NU; ++b) s = fmaf(Q[a][b], sol[b], s);
      sm[S_MK + a] = s + qu[a];
    }
  }
  __syncwarp(wmask);
  // ---- P4: V, v -----------------------------------------------------------
  if (rowx) {
    float2 kc2[NU], qu2[NU];
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      kc2[a] = dup2(Kc[a]);
      qu2[a] = dup2(qxu[a]);
    }
    // column pairs (j, j + 1), column 12 alone
#pragma unroll
    for (int j = 0; j < NX - 1; j += 2) {
      float2 s = make_float2(qxx[j], qxx[j + 1]);
#pragma unroll
      for (int a = 0; a < NU; ++a) s = fma2(kc2[a], ld2(sm + S_M + a * LDM + j), s);
#pragma unroll
      for (int a = 0; a < NU; ++a) s = fma2(qu2[a], ld2(sm + S_K + a * LDM + j), s);
      Vr[j] = s.x;
      Vr[j + 1] = s.y;
    }
    {
      float s = qxx[NX - 1];
#pragma unroll
      for (int a = 0; a < NU; ++a) s = fmaf(Kc[a], sm[S_M + a * LDM + NX - 1], s);
#pragma unroll
      for (int a = 0; a < NU; ++a) s = fmaf(qxu[a], sm[S_K + a * LDM + NX - 1], s);
      Vr[NX - 1] = s;
    }
    float s = qx;
#pragma unroll
    for (int a = 0; a < NU; ++a) s = fmaf(Kc[a], sm[S_MK + a], s);
#pragma unroll
    for (int a = 0; a < NU; ++a) s = fmaf(qxu[a], sm[S_KF + a], s);
    vi = s;
#pragma unroll
    for (int j = 0; j < NX; ++j) sm[S_V + g * LDM + j] = Vr[j];
    sm[S_VV + g] = vi;
  }
  return fb;
}

// Lane g writes row g of A_t, B_t (state-row lanes) at the state and control
// z = [x_t (13); u_t (4)].
__device__ __forceinline__ void jacobian_rows(float* sm, const float* z, int g, float dt) {
  if (g < NX) jac_row(g, z, z + NX, dt, sm + S_A + g * LDM, sm + S_B + g * NU);
}

// v[i] for a lane-dependent i, without a dynamically indexed local array.
template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int i) {
  float r = v[0];
#pragma unroll
  for (int j = 1; j < N; ++j) r = (i == j) ? v[j] : r;
  return r;
}

}  // namespace

// ---------------------------------------------------------------------------
// Solve (controller.py:303-435)
// ---------------------------------------------------------------------------
// MINB: resident one-warp CTAs per SM the register budget targets. 8 (255
// registers, no spills) is faster while the grid fits one wave at 8 CTAs per
// SM; beyond that 12 (168 registers, some spills) is, by the extra warps per
// SM.
template <int MINB>
__global__ void __launch_bounds__(S_THREADS, MINB) dense_solve_kernel(DenseSolveParams p) {
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int e = lane >> 4;   // element slot of the warp
  const int g = lane & 15;   // lane in the group
  const int64_t b = ((int64_t)blockIdx.x * S_WPC + warp) * EPW + e;
  const bool valid = b < p.B;
  const int64_t bw = valid ? b : 0;  // a valid element for address formation
  float* sm = smem + (warp * EPW + e) * S_ELEM;
  const unsigned FULLW = 0xffffffffu;
  const int gbase = lane & 16;
  const int T = p.T;
  const float dt = p.dt;
  const bool rowx = g < NX;
  const float* lo = p.has_bounds ? p.u_min : nullptr;
  const float* hi = p.has_bounds ? p.u_max : nullptr;
  Ws W{p.ws + bw * p.ws_fields, T, p.n_alpha + 1};
  // step t's cost block and linear term (batch-major or time-major layout)
  const int64_t cbs = p.cost_bstride, cts = p.cost_tstride;
  auto Cstep = [&](int t) { return p.C + (bw * cbs + (int64_t)t * cts) * (NT * NT); };
  auto cstep = [&](int t) { return p.c + (bw * cbs + (int64_t)t * cts) * NT; };
  const float* Cf = p.C_f ? p.C_f + bw * NT * NT : nullptr;
  const float* cf = p.c_f ? p.c_f + bw * NT : nullptr;
  const float* xr = p.x_ref ? p.x_ref + bw * (int64_t)(T + 1) * NX : nullptr;
  const float* ur = p.u_ref ? p.u_ref + bw * (int64_t)T * NU : nullptr;
  auto xref = [&](int t, int i) { return xr ? __ldg(xr + t * NX + i) : 0.0f; };
  auto uref = [&](int t, int a) { return ur ? __ldg(ur + t * NU + a) : 0.0f; };

  if (p.trace != nullptr && valid && g == 0)
    for (int i = 0; i < p.max_iter; ++i) p.trace[b * p.max_iter + i] = (int8_t)-128;

  // ---- rollouts: the initial one (controller.py:307-313, lane 0 of the
  // group, controls U_init) and the line search's (controller.py:360-388,
  // 437-533, lane j = step size j). All 16 lanes stage step t + 1 (costs,
  // references, nominal record, gains) into shared memory while the
  // candidate lanes roll out step t from the staged copy.
  const int nsc = L_NSC;
  // n_cand candidates, lanes_per_candidate(n_cand) lanes each: every lane of
  // candidate j rolls it out (identical arithmetic) and costs its share of
  // the rows of the quadratic form; the shares are summed at the end.
  auto rollout = [&](bool init, int nomslot, int n_cand) -> float {
    const int lpc = lanes_per_candidate(n_cand);
    const int j = g / lpc, rsub = g - j * lpc;
    const bool cand = valid && j < n_cand;
    const bool lead = cand && rsub == 0;  // stores the records, adds the linear and terminal terms
    const int cs = init ? 0 : (j < nomslot ? j : j + 1);
    float al = p.alphas[0];
#pragma unroll
    for (int jj = 1; jj < ILQR_MAX_ALPHAS_DEV; ++jj) al = (j == jj) ? p.alphas[jj] : al;
    float* ts = sm + S_TAU + g * NT;
    // step t's inputs go to buffer t & 1 by cp.async, issued one step ahead
    auto buf = [&](int t) { return (t & 1) ? sm + S_LS2 : sm; };
    auto stage = [&](int t) {
      if (!valid) return;
      float* st = buf(t);
#pragma unroll
      for (int k = 0; k < L_PF; ++k) {
        const int f = g + GL * k;
        if (f < L_CV) {
          cp_async4(st + f, Cstep(t) + f);
        } else if (f < L_XR) {
          cp_async4(st + f, cstep(t) + (f - L_CV));
        } else if (f < L_UR) {
          if (xr) cp_async4(st + f, xr + t * NX + (f - L_XR));
          else st[f] = 0.0f;
        } else if (f < L_U0) {
          if (ur) cp_async4(st + f, ur + t * NU + (f - L_UR));
          else st[f] = 0.0f;
        } else if (f < nsc && init) {
          cp_async4(st + f, p.U_init + (b * T + t) * NU + (f - L_U0));
        }
      }
      if (!init) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int q = g + GL * k;
          if (q < L_NF4)
            cp_async16(st + L_F4 + 4 * q, q < 5 ? (const void*)(W.rec(nomslot, t) + q) : (const void*)W.kcol(t, q - 5));
        }
      }
    };
    float x[NX];
    if (cand) {
#pragma unroll
      for (int i = 0; i < NX; ++i) x[i] = __ldg(p.x0 + b * NX + i);
    }
    float sq = 0.0f, sl = 0.0f;
    stage(0);
    cp_async_commit();
    for (int t = 0; t < T; ++t) {
      __syncwarp();  // every lane is done with buffer (t + 1) & 1 (step t - 1)
      if (t + 1 < T) {
        stage(t + 1);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      const float* st = buf(t);
      if (cand) {
        float u[NU];
        if (init) {
#pragma unroll
          for (int a = 0; a < NU; ++a) u[a] = st[L_U0 + a];
        } else {
          float xb[NX], ub[NU];
          load_rec(reinterpret_cast<const float4*>(st + L_F4), xb, ub);
          const float4* kc = reinterpret_cast<const float4*>(st + L_F4) + 5;
          float dx[NX];
#pragma unroll
          for (int j = 0; j < NX; ++j) dx[j] = x[j] - xb[j];
          float kd[NU];
          {
            const float4 c = kc[0];
            kd[0] = c.x * dx[0];
            kd[1] = c.y * dx[0];
            kd[2] = c.z * dx[0];
            kd[3] = c.w * dx[0];
          }
#pragma unroll
          for (int j = 1; j < NX; ++j) {
            const float4 c = kc[j];
            kd[0] = fmaf(c.x, dx[j], kd[0]);
            kd[1] = fmaf(c.y, dx[j], kd[1]);
            kd[2] = fmaf(c.z, dx[j], kd[2]);
            kd[3] = fmaf(c.w, dx[j], kd[3]);
          }
          const float4 k4 = kc[NX];
          const float kt[NU] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int a = 0; a < NU; ++a) {
            float v = ub[a] + (al * kt[a] + al * kd[a]);
            if (lo != nullptr) v = clampn(v, __ldg(lo + a), __ldg(hi + a));
            u[a] = v;
          }
        }
        if (lead) store_rec(W.rec(cs, t), x, u);
        float tau[NT];
#pragma unroll
        for (int i = 0; i < NX; ++i) tau[i] = x[i] - st[L_XR + i];
#pragma unroll
        for (int a = 0; a < NU; ++a) tau[NX + a] = u[a] - st[L_UR + a];
#pragma unroll
        for (int i = 0; i < NT; ++i) ts[i] = tau[i];
        sq += step_quad_rows(st, tau, ts, rsub, lpc);
        if (lead) {
          float l = st[L_CV] * tau[0];
#pragma unroll
          for (int jj = 1; jj < NT; ++jj) l = fmaf(st[L_CV + jj], tau[jj], l);
          sl += l;
        }
        float xn[NX];
        step(x, u, dt, xn);
#pragma unroll
        for (int i = 0; i < NX; ++i) x[i] = xn[i];
      }
    }
    // the candidate's row shares, in sub-lane order
    const int base = (lane & 16) + j * lpc;
    float sqa = __shfl_sync(FULLW, sq, base & 31);
    for (int k = 1; k < 4; ++k) {
      const float v = __shfl_sync(FULLW, sq, (base + k) & 31);
      if (k < lpc) sqa += v;
    }
    float cost = 0.0f;
    if (lead) {
      const float zu[NU] = {0.0f, 0.0f, 0.0f, 0.0f};
      store_rec(W.rec(cs, T), x, zu);
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = x[i] - xref(T, i);
      cost = (0.5f * sqa + sl) + terminal_cost(Cf, cf, tn);
    }
    __syncwarp();
    return cost;
  };

  float best = rollout(true, 0, 1);
  best = __shfl_sync(FULLW, best, gbase);

  uint32_t status = 0;
  bool active = valid;
  int iters = 0;
  int stall_iter = p.max_iter;
  float stall_gap = 0.0f;
  int nom = 0;

  for (int it = 0; it < p.max_iter; ++it) {
    if (p.forced != nullptr && active && p.forced[b * p.max_iter + it] == (int8_t)-128) active = false;
    if (!__any_sync(FULLW, active)) break;

    // ---- backward Riccati pass (controller.py:315-318, 697-723) ------------
    float Vr[NX], vi = 0.0f, Kc[NU], kf[NU];
    {
      if (g < 5) reinterpret_cast<float4*>(sm + S_Z)[g] = W.rec(nom, T)[g];
      __syncwarp();
      if (rowx) {
        float tn[NX];
#pragma unroll
        for (int j = 0; j < NX; ++j) tn[j] = sm[S_Z + j] - xref(T, j);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NX; ++j) {
          Vr[j] = Cf ? __ldg(Cf + g * NT + j) : 0.0f;
          s = fmaf(Vr[j], tn[j], s);
        }
        vi = s + (cf ? __ldg(cf + g) : 0.0f);
#pragma unroll
        for (int j = 0; j < NX; ++j) sm[S_V + g * LDM + j] = Vr[j];
        sm[S_VV + g] = vi;
      }
    }
    bool fallback = false;
    for (int t = T - 1; t >= 0; --t) {
      __syncwarp();
      if (g < 5) reinterpret_cast<float4*>(sm + S_Z)[g] = W.rec(nom, t)[g];
      __syncwarp();
      jacobian_rows(sm, sm + S_Z, g, dt);
      // l_tau = C tau + c for this lane's rows (cost.py:130-171)
      float tau[NT];
#pragma unroll
      for (int i = 0; i < NX; ++i) tau[i] = sm[S_Z + i] - xref(t, i);
#pragma unroll
      for (int a = 0; a < NU; ++a) tau[NX + a] = sm[S_Z + NX + a] - uref(t, a);
      const float* Ct = Cstep(t);
      const float* ct = cstep(t);
      StepIn in;
      in.lx = 0.0f;
      in.lu = 0.0f;
      if (rowx) {
        const float* row = Ct + g * NT;
        float crow[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) crow[j] = __ldg(row + j);
        float s = crow[0] * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) s = fmaf(crow[j], tau[j], s);
        in.lx = s + __ldg(ct + g);
#pragma unroll
        for (int j = 0; j < NX; ++j) in.cxx[j] = crow[j];
#pragma unroll
        for (int a = 0; a < NU; ++a) in.cxu[a] = crow[NX + a];
      }
      if (g < NU) {
        const float* row = Ct + (NX + g) * NT;
        float s = __ldg(row) * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) s = fmaf(__ldg(row + j), tau[j], s);
        in.lu = s + __ldg(ct + NX + g);
      }
      in.cuu = __ldg(Ct + (NX + (g >> 2)) * NT + NX + (g & 3));
      __syncwarp();
      const bool fb = riccati_step<false>(sm, g, rowx, valid, FULLW, in, p.reg, nullptr, Vr, vi, Kc, kf);
      fallback |= fb;
      if (valid) {
        if (rowx) *W.kcol(t, g) = make_float4(Kc[0], Kc[1], Kc[2], Kc[3]);
        if (g == NX) *W.kff(t) = make_float4(kf[0], kf[1], kf[2], kf[3]);
      }
    }
    if (fallback && active) status |= ELEM_CHOL_FALLBACK;
    __syncwarp();

    // ---- grid line search (controller.py:360-388, 437-533): lane j = step j --
    const float mine = rollout(false, nom, p.n_alpha);
    const int lpc_ls = lanes_per_candidate(p.n_alpha);
    // torch.argmin semantics over the step sizes: first NaN, else first minimum
    int jbest = 0;
    float cmin = 0.0f;
    bool have = false, nan_seen = false;
    float cand[ILQR_MAX_ALPHAS_DEV];
#pragma unroll
    for (int jj = 0; jj < ILQR_MAX_ALPHAS_DEV; ++jj) {
      const float cj = __shfl_sync(FULLW, mine, (gbase + jj * lpc_ls) & 31);
      cand[jj] = cj;
      if (jj >= p.n_alpha) continue;
      if (!nan_seen) {
        if (cj != cj) {
          nan_seen = true;
          jbest = jj;
          cmin = cj;
        } else if (!have || cj < cmin) {
          have = true;
          jbest = jj;
          cmin = cj;
        }
      }
    }

    // ---- decision (controller.py:396-415) ---------------------------------
    if (active) {
      bool accept;
      int jsel = jbest;
      ++iters;
      if (p.forced != nullptr) {
        const int8_t d = p.forced[b * p.max_iter + it];
        accept = d >= 0 && d < p.n_alpha;
        if (accept) jsel = d;
      } else {
        accept = cmin < best;
      }
      if (p.trace != nullptr && g == 0) p.trace[b * p.max_iter + it] = (int8_t)(accept ? jsel : -(jbest + 1));
      if (!accept && stall_iter == p.max_iter) {
        stall_iter = it;
        stall_gap = fabsf(cmin - best);
      }
      if (accept) {
        float cs = cand[0];
#pragma unroll
        for (int jj = 1; jj < ILQR_MAX_ALPHAS_DEV; ++jj) cs = (jj == jsel) ? cand[jj] : cs;
        best = cs;
        nom = jsel < nom ? jsel : jsel + 1;
      }
      if (!accept && p.forced == nullptr) active = false;
    }
    __syncwarp();
  }

  // ---- outputs ------------------------------------------------------------------
  bool finite = true;
  if (valid) {
    const float* nrec = reinterpret_cast<const float*>(W.rec(nom, 0));
    for (int f = g; f < (T + 1) * NX; f += GL) {
      const int t = f / NX, i = f - t * NX;
      const float xv = nrec[t * REC + i];
      finite &= isfinite(xv);
      p.X[b * (T + 1) * NX + f] = xv;
    }
    for (int f = g; f < T * NU; f += GL) {
      const int t = f / NU, a = f - t * NU;
      const float uv = nrec[t * REC + NX + a];
      finite &= isfinite(uv);
      p.U[b * T * NU + f] = uv;
      if (p.tight != nullptr) {
        // torch.isclose(U, bound, rtol=1e-5, atol=1e-7) against u_min, u_max
        bool tt = false;
        if (lo != nullptr) {
          const float l_ = __ldg(lo + a), h_ = __ldg(hi + a);
          const float e0 = fabsf(uv - l_), e1 = fabsf(uv - h_);
          tt = (uv == l_) || (isfinite(e0) && e0 <= 1e-7f + fabsf(1e-5f * l_)) || (uv == h_) ||
               (isfinite(e1) && e1 <= 1e-7f + fabsf(1e-5f * h_));
        }
        p.tight[b * T * NU + f] = tt ? 1 : 0;
      }
    }
  }
  const bool all_finite = group_sum(finite ? 0.0f : 1.0f, FULLW) == 0.0f;
  if (!all_finite) status |= ELEM_NONFINITE;
  if (valid && g == 0) {
    if (p.iters) p.iters[b] = iters;
    if (p.status) p.status[b] = status;
    if (p.best_cost) p.best_cost[b] = best;
    if (p.stall_iter) p.stall_iter[b] = stall_iter;
    if (p.stall_gap) p.stall_gap[b] = stall_gap;
  }
}

// ---------------------------------------------------------------------------
// Implicit-diff backward (controller.py:68-133, 1006-1131)
// ---------------------------------------------------------------------------
// 4 CTAs per SM (128 registers, 16 B of spills) against 3 (161, none): 4 % faster
// at B=16384, the same for small grids.
__global__ void __launch_bounds__(THREADS, 4) dense_backward_kernel(DenseBackwardParams p) {
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int e = lane >> 4;
  const int g = lane & 15;
  const int64_t b = ((int64_t)blockIdx.x * WPC + warp) * EPW + e;
  const bool valid = b < p.B;
  const int64_t bw = valid ? b : 0;
  float* sm = smem + (warp * EPW + e) * S_ELEM_BWD;
  const unsigned FULLW = 0xffffffffu;
  const int T = p.T;
  const float dt = p.dt;
  const bool rowx = g < NX;
  const float* Xb = p.X + bw * (int64_t)(T + 1) * NX;
  const float* Ub = p.U + bw * (int64_t)T * NU;
  const int64_t cbs = p.cost_bstride, cts = p.cost_tstride;
  auto Cstep = [&](int t) { return p.C + (bw * cbs + (int64_t)t * cts) * (NT * NT); };
  const float* Cf = p.C_f ? p.C_f + bw * NT * NT : nullptr;
  const float* xr = p.x_ref ? p.x_ref + bw * (int64_t)(T + 1) * NX : nullptr;
  const float* gX = p.gX + bw * (int64_t)(T + 1) * NX;
  const float* gU = p.gU + bw * (int64_t)T * NU;
  const uint8_t* tb = p.tight ? p.tight + bw * (int64_t)T * NU : nullptr;
  float4* kws = reinterpret_cast<float4*>(p.ws + bw * (int64_t)T * (NX + 1) * 4);

  // ---- masked adjoint Riccati: V_T = C_f,xx, v_T = -dL/dX_T -------------
  float Vr[NX], vi = 0.0f, Kc[NU], kf[NU];
  if (rowx) {
#pragma unroll
    for (int j = 0; j < NX; ++j) {
      Vr[j] = Cf ? __ldg(Cf + g * NT + j) : 0.0f;
      sm[S_V + g * LDM + j] = Vr[j];
    }
    vi = -__ldg(gX + T * NX + g);
    sm[S_VV + g] = vi;
  }
  // Step t - 1's inputs (C, X, U, dL/dX, dL/dU, tight mask) are copied into
  // the other staging buffer while step t computes.
  auto stage_z = [&](int t, float* st) {
    if (g < NX) cp_async4(st + R_REC + g, Xb + t * NX + g);
    if (g < NU) cp_async4(st + R_REC + NX + g, Ub + t * NU + g);
  };
  auto bwd_stage = [&](int t, float* st) {
    const float* Ct = Cstep(t);
    for (int f = g; f < NT * NT; f += GL) cp_async4(st + R_C + f, Ct + f);
    stage_z(t, st);
    if (g < NX) cp_async4(st + R_GX + g, gX + t * NX + g);
    if (g < NU) cp_async4(st + R_GU + g, gU + t * NU + g);
    if (g == 0) {
      if (tb) cp_async4(st + R_TM, tb + t * NU);
      else reinterpret_cast<uint32_t*>(st)[R_TM] = 0u;
    }
  };
  auto stb = [&](int t) { return sm + S_STG + ((T - 1 - t) & 1) * R_SIZE; };
  bwd_stage(T - 1, stb(T - 1));
  cp_async_commit();
  for (int t = T - 1; t >= 0; --t) {
    if (t > 0) {
      bwd_stage(t - 1, stb(t - 1));
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const float* st = stb(t);
    jacobian_rows(sm, st + R_REC, g, dt);
    StepIn in;
    in.lx = rowx ? -st[R_GX + g] : 0.0f;
    in.lu = g < NU ? -st[R_GU + g] : 0.0f;
    if (rowx) {
#pragma unroll
      for (int j = 0; j < NX; ++j) in.cxx[j] = st[R_C + g * NT + j];
#pragma unroll
      for (int a = 0; a < NU; ++a) in.cxu[a] = st[R_C + g * NT + NX + a];
    }
    in.cuu = st[R_C + (NX + (g >> 2)) * NT + NX + (g & 3)];
    bool tight[NU];
    {
      const uint32_t tw = reinterpret_cast<const uint32_t*>(st)[R_TM];
#pragma unroll
      for (int a = 0; a < NU; ++a) tight[a] = ((tw >> (8 * a)) & 0xffu) != 0u;
    }
    __syncwarp();
    riccati_step<true>(sm, g, rowx, valid, FULLW, in, p.reg, tight, Vr, vi, Kc, kf);
    if (valid) {
      if (rowx) kws[t * (NX + 1) + g] = make_float4(Kc[0], Kc[1], Kc[2], Kc[3]);
      if (g == NX) kws[t * (NX + 1) + NX] = make_float4(kf[0], kf[1], kf[2], kf[3]);
    }
  }
  if (valid && rowx && p.g_x0) p.g_x0[b * NX + g] = -vi;
  __syncwarp();

  // ---- tangent sweep dU = K dX + k, dX+ = A dX + B dU, and the gradients ------
  float* dts = sm + S_M;  // dtau_t = [dX_t; dU_t] (17)
  if (rowx) dts[g] = 0.0f;
  // Step t + 1's X, U and K_t columns are copied into the other staging
  // buffer while step t computes (the gains were written by this warp's
  // lanes in the pass above; cp.async.cg reads them from L2).
  auto sweep_stage = [&](int t, float* st) {
    stage_z(t, st);
    if (g < NX + 1) {
      float4* d4 = reinterpret_cast<float4*>(st + R_C) + g;
      if (valid) cp_async16(d4, kws + t * (NX + 1) + g);
      else *d4 = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto sb = [&](int t) { return sm + S_STG + (t & 1) * R_SIZE; };
  __syncwarp();
  sweep_stage(0, sb(0));
  cp_async_commit();
  for (int t = 0; t < T; ++t) {
    if (t + 1 < T) {
      sweep_stage(t + 1, sb(t + 1));
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const float* st = sb(t);
    jacobian_rows(sm, st + R_REC, g, dt);
    float dx[NX];
#pragma unroll
    for (int j = 0; j < NX; ++j) dx[j] = dts[j];
    float du[NU];
    {
      const float4* kc = reinterpret_cast<const float4*>(st + R_C);
      const float4 c0 = kc[0];
      float kd[NU] = {c0.x * dx[0], c0.y * dx[0], c0.z * dx[0], c0.w * dx[0]};
#pragma unroll
      for (int j = 1; j < NX; ++j) {
        const float4 c = kc[j];
        kd[0] = fmaf(c.x, dx[j], kd[0]);
        kd[1] = fmaf(c.y, dx[j], kd[1]);
        kd[2] = fmaf(c.z, dx[j], kd[2]);
        kd[3] = fmaf(c.w, dx[j], kd[3]);
      }
      const float4 k4 = kc[NX];
      du[0] = kd[0] + k4.x;
      du[1] = kd[1] + k4.y;
      du[2] = kd[2] + k4.z;
      du[3] = kd[3] + k4.w;
    }
    if (g < NU) dts[NX + g] = pick(du, g);
    // dX_{t+1}, row g (A_t row g was written by this lane)
    float dxn = 0.0f;
    if (rowx) {
      float s = sm[S_A + g * LDM] * dx[0];
#pragma unroll
      for (int k = 1; k < NX; ++k) s = fmaf(sm[S_A + g * LDM + k], dx[k], s);
      float sb = sm[S_B + g * NU] * du[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) sb = fmaf(sm[S_B + g * NU + a], du[a], sb);
      dxn = s + sb;
    }
    __syncwarp();
    if (valid) {
      // dtau = [dX_t; dU_t], z = [X_t; U_t]:
      // grad_C_t = -1/2 (dtau z^T + z dtau^T), grad_c_t = -dtau
      const int64_t off = (b * cbs + (int64_t)t * cts) * NT;
      const float* z = st + R_REC;
      auto grad_row = [&](int i, float* gC) {
        const float dzi = dts[i], zi = z[i];
#pragma unroll
        for (int j = 0; j < NT; ++j) gC[i * NT + j] = -0.5f * (dzi * z[j] + zi * dts[j]);
      };
      if (p.g_C) {
        float* gC = p.g_C + off * NT;
        if (rowx) grad_row(g, gC);
        if (g < NU) grad_row(NX + g, gC);
      }
      if (p.g_c) {
        if (rowx) p.g_c[off + g] = -dts[g];
        if (g < NU) p.g_c[off + NX + g] = -dts[NX + g];
      }
      if (p.g_xref && rowx) p.g_xref[(b * (T + 1) + t) * NX + g] = dts[g];
      if (p.g_uref && g < NU) p.g_uref[(b * T + t) * NU + g] = dts[NX + g];
    }
    __syncwarp();
    if (rowx) dts[g] = dxn;
  }
  __syncwarp();
  if (valid) {
    // terminal: grad_C_final xx = -1/2 (dX_T e^T + e dX_T^T), e = X_T - x_ref_T
    auto eT = [&](int j) { return __ldg(Xb + T * NX + j) - (xr ? __ldg(xr + T * NX + j) : 0.0f); };
    if (p.g_xref && rowx) p.g_xref[(b * (T + 1) + T) * NX + g] = 0.0f;
    if (p.g_Cf) {
      float* gCf = p.g_Cf + b * NT * NT;
      if (rowx) {
        const float dg = dts[g], eg = eT(g);
#pragma unroll
        for (int j = 0; j < NT; ++j) gCf[g * NT + j] = j < NX ? -0.5f * (dg * eT(j) + eg * dts[j]) : 0.0f;
      }
      if (g < NU) {
#pragma unroll
        for (int j = 0; j < NT; ++j) gCf[(NX + g) * NT + j] = 0.0f;
      }
    }
    if (p.g_cf) {
      if (rowx) p.g_cf[b * NT + g] = -dts[g];
      if (g < NU) p.g_cf[b * NT + NX + g] = 0.0f;
    }
  }
}

// One model step / Jacobian per thread (component checks and callers that
// want the model alone).
__global__ void rotor13_dynamics_kernel(const float* __restrict__ x, const float* __restrict__ u, int64_t n,
                                        float dt, float* __restrict__ xn) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xv[NX], uv[NU], out[NX];
#pragma unroll
  for (int j = 0; j < NX; ++j) xv[j] = __ldg(x + i * NX + j);
#pragma unroll
  for (int j = 0; j < NU; ++j) uv[j] = __ldg(u + i * NU + j);
  step(xv, uv, dt, out);
#pragma unroll
  for (int j = 0; j < NX; ++j) xn[i * NX + j] = out[j];
}

// Thread per (element, step, row): row r of A [B,T,13,13] and B [B,T,13,4].
__global__ void rotor13_linearize_kernel(const float* __restrict__ X, const float* __restrict__ U, int64_t B,
                                         int T, float dt, float* __restrict__ A, float* __restrict__ Bm) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * T * NX) return;
  const int r = (int)(idx % NX);
  const int64_t bt = idx / NX;
  const int64_t b = bt / T;
  const int t = (int)(bt - b * T);
  float xv[NX], uv[NU], a[NX], bb[NU];
#pragma unroll
  for (int j = 0; j < NX; ++j) xv[j] = __ldg(X + (b * (T + 1) + t) * NX + j);
#pragma unroll
  for (int j = 0; j < NU; ++j) uv[j] = __ldg(U + bt * NU + j);
  jac_row(r, xv, uv, dt, a, bb);
#pragma unroll
  for (int j = 0; j < NX; ++j) A[(bt * NX + r) * NX + j] = a[j];
#pragma unroll
  for (int j = 0; j < NU; ++j) Bm[(bt * NX + r) * NU + j] = bb[j];
}

}  // namespace r13

int64_t dense_solve_ws_fields(int T, int n_alpha) {
  return (int64_t)(n_alpha + 1) * (T + 1) * r13::REC + (int64_t)T * (r13::NX + 1) * 4;
}

int64_t dense_backward_ws_fields(int T) { return (int64_t)T * (r13::NX + 1) * 4; }

static size_t dense_smem_bytes(int elem_floats) { return (size_t)r13::EPC * elem_floats * sizeof(float); }

cudaError_t launch_dense_solve(const DenseSolveParams& p, cudaStream_t stream) {
  if (p.B == 0) return cudaSuccess;
  const int64_t grid = (p.B + r13::S_EPC - 1) / r13::S_EPC;
  const size_t smem = (size_t)r13::S_EPC * r13::S_ELEM * sizeof(float);
  if (grid > 8 * r13::SM_COUNT)
    r13::dense_solve_kernel<12><<<(unsigned)grid, r13::S_THREADS, smem, stream>>>(p);
  else
    r13::dense_solve_kernel<8><<<(unsigned)grid, r13::S_THREADS, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_dense_backward(const DenseBackwardParams& p, cudaStream_t stream) {
  if (p.B == 0) return cudaSuccess;
  // more than the default 48 KB of dynamic shared memory per CTA
  cudaError_t e = cudaFuncSetAttribute(r13::dense_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)dense_smem_bytes(r13::S_ELEM_BWD));
  if (e != cudaSuccess) return e;
  const int64_t grid = (p.B + r13::EPC - 1) / r13::EPC;
  r13::dense_backward_kernel<<<(unsigned)grid, r13::THREADS, dense_smem_bytes(r13::S_ELEM_BWD), stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_rotor13_dynamics(const float* x, const float* u, int64_t n, float dt, float* xn,
                                    cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  r13::rotor13_dynamics_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, u, n, dt, xn);
  return cudaGetLastError();
}

cudaError_t launch_rotor13_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A,
                                     float* Bm, cudaStream_t s) {
  const int64_t n = B * T * r13::NX;
  if (n == 0) return cudaSuccess;
  r13::rotor13_linearize_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(X, U, B, T, dt, A, Bm);
  return cudaGetLastError();
}

}  // namespace ilqr
