// ilqr_team.cuh -- one batch element per 5-lane team (6 elements per warp).
//
// Riccati step: lane m of a team owns two state rows of V, RA(m) and RB(m):
//   RA = {3,4,5,6,0}  (the four quaternion rows, and p0)
//   RB = {1,2,7,8,9}  (p1, p2 and the three velocity rows)
// so that every lane runs the same instruction stream: for its RA row it
// applies an 8-term combination over rows {3..9, own} of (V A) (the column of A
// at a quaternion row has nonzeros exactly there; for p0 only the own-row
// coefficient is 1), and for its RB row a 2-term combination (own row plus dt
// times p_j for a velocity row, 0 for a position row). Terms with an exact
// zero coefficient add exact zeros, so the result equals the structured sum.
// Rows of V A, V B, v, K and Q_xu are exchanged through a per-element
// shared-memory area; everything else stays in registers.
//
// Line search: lane m evaluates step size alpha_m (5 at a time).
#pragma once

#include "ilqr_device.cuh"
#include "ilqr_kernels.h"

namespace ilqr {

constexpr int TEAM = 5;
constexpr int EPW = 6;        // batch elements per warp
constexpr int XS = 180;       // exchange floats per element (180 = 20 mod 32: bank spread)
// exchange layout (floats). V B, v and l_u are dead once the gains are solved
// (a warp sync separates the phases); K and Q_xu rows take their place while
// the V A rows stay for the value update.
constexpr int X_VA = 0;       // [10][10] rows of V A
constexpr int X_VB = 100;     // [10][4]  rows of V B
constexpr int X_V = 140;      // [10]     v
constexpr int X_LU = 152;     // [4]      l_u
constexpr int X_K = 100;      // [4][10]  K: gain row a at X_K + 10a (over V B)
constexpr int X_QXU = 140;    // [4][10]  Q_ux: Q_xu[c][a] at X_QXU + 10a + c (over v, l_u)
constexpr uint32_t TSLAB_BYTES = EPW * CBLK * 4u;  // bytes one TMA box delivers

// Register tiers: minimum residencies (CTAs of one warp per SM) the kernels
// are compiled for. 19 CTAs per SM caps registers at 96 (one scheduler holds
// five warps of its 16 K registers), 12 at 168, 8 at 255; fewer registers
// spill. The launch takes the fattest tier whose residency fits the grid in
// one wave, except where more waves of a fatter tier are faster (B200,
// T = 20, 5 iterations):
//  - The solve's 96-register build spills across every Riccati step. Past
//    1.5 waves of the 12-CTA tier (B > 15984) that tier is faster than one
//    19-CTA wave (B = 14336: 2.2 % slower, 15360: even, 16384: 2.7 % faster),
//    and past one 19-CTA wave by far (B = 20480: 1.34 against 1.98 ms;
//    B = 65536: 13 %).
//  - The backward spills less at 96 registers: it takes the 19-CTA tier up
//    to one wave (B = 16384: 0.245 against 0.259 ms at 12 CTAs) and the
//    12-CTA tier beyond (B = 20480: 0.280 against 0.383 ms; B = 65536: 2.5 %).
constexpr int SMS = 148;
constexpr int TIER_LO = 19, TIER_MID = 12, TIER_HI = 8;
inline int pick_solve_tier(int64_t grid) {
  if (grid <= (int64_t)SMS * TIER_HI) return TIER_HI;
  if (grid <= (int64_t)SMS * TIER_MID) return TIER_MID;
  return 2 * grid <= 3 * (int64_t)SMS * TIER_MID ? TIER_LO : TIER_MID;
}
inline int pick_backward_tier(int64_t grid) {
  if (grid <= (int64_t)SMS * TIER_HI) return TIER_HI;
  if (grid <= (int64_t)SMS * TIER_MID) return TIER_MID;
  return grid <= (int64_t)SMS * TIER_LO ? TIER_LO : TIER_MID;
}

__device__ __forceinline__ int row_a(int m) { return m < 4 ? 3 + m : 0; }

__device__ __forceinline__ int row_b(int m) { return m == 0 ? 1 : (m == 1 ? 2 : 5 + m); }

// Offset of entry i (tau order: p 0..2, q 3..6, v 7..9, thrust 10, w 11..13)
// of step t within the x_q half of a sigmoid cost row (the x_p half adds 14 T).
// _build_cost_tensors (training_modules/mlp_mpc_policy_diffmpc.py:194-247)
// slices x_q into blocks of T steps: p (3), q (4), v (3), w (3), thrust (1).
__device__ __forceinline__ int sig_off(int T, int t, int i) {
  if (i < 3) return 3 * t + i;
  if (i < 7) return 3 * T + 4 * t + (i - 3);
  if (i < 10) return 7 * T + 3 * t + (i - 7);
  if (i == 10) return 13 * T + t;
  return 10 * T + 3 * t + (i - 11);
}

// diag(C_t)_i and c_t,i from a sigmoid cost row q (fp32, the reference's
// operation order: one multiply, then one add or subtract).
__device__ __forceinline__ float sig_diag(const SigmoidCost& s, const float* q, int T, int t, int i) {
  return __ldg(q + sig_off(T, t, i)) * s.range_q + s.eps;
}
__device__ __forceinline__ float sig_c(const SigmoidCost& s, const float* q, int T, int t, int i) {
  const float x = __ldg(q + 14 * T + sig_off(T, t, i));
  return i == NX ? -(x * s.range_pt + s.eps) : (x - 0.5f) * s.range_p;
}

// Access to one element's C_t block in shared memory.
struct DenseC {
  const float* Ct;
  __device__ __forceinline__ float operator()(int i, int j) const { return Ct[i * NT + j]; }
  // entries (i, j) and (i, j + 1); j even (8-byte aligned: NT is even)
  __device__ __forceinline__ float2 pair(int i, int j) const { return ld2(Ct + i * NT + j); }
};

// Coefficients A[k][RA] for k = 3..9 and the own-row coefficient, for lane m.
__device__ __forceinline__ void coef_a(const Jac& J, int m, float (&c)[8]) {
  const float z = 0.0f;
  // columns j of A[q][q] and A[v][q] (see the table in ilqr_device.cuh)
  if (m == 0) {
    c[0] = 1.0f; c[1] = J.h0; c[2] = J.h1; c[3] = J.h2; c[4] = J.g2; c[5] = -J.g1; c[6] = J.g0;
  } else if (m == 1) {
    c[0] = -J.h0; c[1] = 1.0f; c[2] = -J.h2; c[3] = J.h1; c[4] = J.g3; c[5] = -J.g0; c[6] = -J.g1;
  } else if (m == 2) {
    c[0] = -J.h1; c[1] = J.h2; c[2] = 1.0f; c[3] = -J.h0; c[4] = J.g0; c[5] = J.g3; c[6] = -J.g2;
  } else if (m == 3) {
    c[0] = -J.h2; c[1] = -J.h1; c[2] = J.h0; c[3] = 1.0f; c[4] = J.g1; c[5] = J.g2; c[6] = J.g3;
  } else {
    c[0] = z; c[1] = z; c[2] = z; c[3] = z; c[4] = z; c[5] = z; c[6] = z;
  }
  c[7] = (m == 4) ? 1.0f : z;
}

// Row [own | V] (A) -> (V A)[r][:] and (V B)[r][:] for one row r of V.
__device__ __forceinline__ void row_VA_VB(const Jac& J, const float (&Vr)[NX], float (&va)[NX], float (&vb)[NU]) {
#pragma unroll
  for (int j = 0; j < 3; ++j) va[j] = Vr[j];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float acc = Vr[3] * aqq(J, 0, j);
#pragma unroll
    for (int mm = 1; mm < 4; ++mm) acc = fmaf(Vr[3 + mm], aqq(J, mm, j), acc);
#pragma unroll
    for (int n = 0; n < 3; ++n) acc = fmaf(Vr[7 + n], avq(J, n, j), acc);
    va[3 + j] = acc;
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) va[7 + j] = fmaf(Vr[j], J.dt, Vr[7 + j]);
  {
    float acc = Vr[7] * J.bv0;
    acc = fmaf(Vr[8], J.bv1, acc);
    vb[0] = fmaf(Vr[9], J.bv2, acc);
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    float acc = Vr[3] * bqw(J, 0, k);
#pragma unroll
    for (int mm = 1; mm < 4; ++mm) acc = fmaf(Vr[3 + mm], bqw(J, mm, k), acc);
    vb[1 + k] = acc;
  }
}

// One Riccati step for a team.
// Forward (MASKED=false), backward_lqr (DifferentialMPC/controller.py:697-723):
//   Q_xx = l_xx + A^T V A          Q_xu = l_xu + A^T V B
//   Q_uu = l_uu + B^T V B + reg I
//   q_x = l_x + A^T v              q_u = l_u + B^T v
//   [K | k] = -chol_solve(Q_uu + reg I, [Q_ux | q_u])   (reg added twice)
//   V = Q_xx + (K^T Q_uu + Q_xu) K + K^T Q_ux
//   v = q_x + (K^T Q_uu + Q_xu) k + K^T q_u
// Backward (MASKED=true), _zero_constrained_lqr (controller.py:1035-1110):
//   tight rows/cols of Q_uu zeroed, +1 on their diagonal, + (1e-8 reg) I;
//   tight rows of Q_ux and entries of q_u zeroed for the solve only;
//   V, v use the unmasked Q_uu, Q_ux, q_u, and v = q_x + K^T(Q_uu k + q_u) + Q_xu k.
// Va, Vb: this lane's rows RA, RB of V (in V_{t+1}, out V_t); va_, vb_: the
// matching entries of v. lxa, lxb: gradient terms of those rows; the four
// control gradient terms are read from xc[X_LU..] (written by lanes 0..3
// before the call). live: the lane's team owns a batch element. xc: this
// element's exchange area. Ct: this element's C_t block in shared memory
// (DenseC). after_c() is called at the end, once every lane is done reading
// Ct and the exchange area (it may reuse the slab); it must sync the warp. Outputs: Ka, Kb = K[:, RA],
// K[:, RB]; k. Returns false if the Cholesky failed (SVD inverse used).
template <bool MASKED, bool STRAIGHT, class CAcc, class AfterC>
__device__ __forceinline__ bool team_riccati(float (&Va)[NX], float (&Vb)[NX], float& va_, float& vb_,
                                             const Jac& J, const CAcc& Ct, float lxa, float lxb,
                                             float reg, uint32_t tight, int m, bool live,
                                             float* __restrict__ xc, AfterC&& after_c, float (&Ka)[NU],
                                             float (&Kb)[NU], float (&k)[NU]) {
  const int ra = row_a(m), rb = row_b(m);
  // ---- rows of V A and V B -> exchange ------------------------------------
  {
    float VAr[NX], VBr[NU];
    row_VA_VB(J, Va, VAr, VBr);
#pragma unroll
    for (int c = 0; c < NX; c += 2)
      *reinterpret_cast<float2*>(xc + X_VA + ra * NX + c) = make_float2(VAr[c], VAr[c + 1]);
    *reinterpret_cast<float4*>(xc + X_VB + ra * NU) = make_float4(VBr[0], VBr[1], VBr[2], VBr[3]);
    row_VA_VB(J, Vb, VAr, VBr);
#pragma unroll
    for (int c = 0; c < NX; c += 2)
      *reinterpret_cast<float2*>(xc + X_VA + rb * NX + c) = make_float2(VAr[c], VAr[c + 1]);
    *reinterpret_cast<float4*>(xc + X_VB + rb * NU) = make_float4(VBr[0], VBr[1], VBr[2], VBr[3]);
  }
  xc[X_V + ra] = va_;
  xc[X_V + rb] = vb_;
  __syncwarp();

  // ---- Q_xu rows and q_x entries of my rows, Q_uu and q_u -----------------
  float ca[8];
  coef_a(J, m, ca);
  const float cb = (m >= 2) ? J.dt : 0.0f;
  const int pb = (m >= 2) ? m - 2 : 0;
  // Coefficients as packed pairs (the same value in both halves): every
  // product below pairs two columns of one row.
  float2 c2[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) c2[s] = dup2(ca[s]);
  const float2 cb2 = dup2(cb);
  float Qxa[NU], Qxb[NU], qxa, qxb;
  {
    // RA: sum over rows 3..9 of V B (and v), then the own row.
    float2 acc01 = make_float2(0.0f, 0.0f), acc23 = make_float2(0.0f, 0.0f);
    float accv = 0.0f;
#pragma unroll
    for (int s = 0; s < 7; ++s) {
      const float* r = xc + X_VB + (3 + s) * NU;
      acc01 = fma2(c2[s], ld2(r), acc01);
      acc23 = fma2(c2[s], ld2(r + 2), acc23);
      accv = fmaf(ca[s], xc[X_V + 3 + s], accv);
    }
    {
      const float* own = xc + X_VB + ra * NU;
      const float2 q01 = add2(Ct.pair(ra, NX), fma2(c2[7], ld2(own), acc01));
      const float2 q23 = add2(Ct.pair(ra, NX + 2), fma2(c2[7], ld2(own + 2), acc23));
      Qxa[0] = q01.x; Qxa[1] = q01.y; Qxa[2] = q23.x; Qxa[3] = q23.y;
    }
    qxa = lxa + fmaf(ca[7], va_, accv);
    // RB: own row plus cb times row pb.
    {
      const float* pr = xc + X_VB + pb * NU;
      const float* own = xc + X_VB + rb * NU;
      const float2 q01 = add2(Ct.pair(rb, NX), fma2(cb2, ld2(pr), ld2(own)));
      const float2 q23 = add2(Ct.pair(rb, NX + 2), fma2(cb2, ld2(pr + 2), ld2(own + 2)));
      Qxb[0] = q01.x; Qxb[1] = q01.y; Qxb[2] = q23.x; Qxb[3] = q23.y;
    }
    qxb = lxb + fmaf(cb, xc[X_V + pb], vb_);
  }
  float Quu[NU][NU], qu[NU];
  {
    // Q_uu = l_uu + B^T (V B) + reg I: B^T rows are bv over the velocity rows
    // (first control) and 0.5 dt Xi(q) over the quaternion rows (body rates);
    // accumulated row by row of V B in index order.
    // (columns paired: acc[a][h] holds columns 2h, 2h + 1 of row a)
    float2 acc[NU][2];
#pragma unroll
    for (int s = 0; s < 7; ++s) {
      const float* r = xc + X_VB + (3 + s) * NU;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 rh = ld2(r + 2 * h);
        if (s >= 4) {
          const float2 cf = dup2(bvf(J, s - 4));
          acc[0][h] = (s == 4) ? mul2(cf, rh) : fma2(cf, rh, acc[0][h]);
        } else {
#pragma unroll
          for (int kk = 0; kk < 3; ++kk) {
            const float2 cf = dup2(bqw(J, s, kk));
            acc[1 + kk][h] = (s == 0) ? mul2(cf, rh) : fma2(cf, rh, acc[1 + kk][h]);
          }
        }
      }
    }
#pragma unroll
    for (int a = 0; a < NU; ++a)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 rg = make_float2(a == 2 * h ? reg : 0.0f, a == 2 * h + 1 ? reg : 0.0f);
        const float2 q = add2(add2(Ct.pair(NX + a, NX + 2 * h), acc[a][h]), rg);
        Quu[a][2 * h] = q.x;
        Quu[a][2 * h + 1] = q.y;
      }
    float vq[7];
#pragma unroll
    for (int s = 0; s < 7; ++s) vq[s] = xc[X_V + 3 + s];
    float lu[NU];
#pragma unroll
    for (int a = 0; a < NU; ++a) lu[a] = xc[X_LU + a];
    {
      float acc = J.bv0 * vq[4];
      acc = fmaf(J.bv1, vq[5], acc);
      qu[0] = lu[0] + fmaf(J.bv2, vq[6], acc);
#pragma unroll
      for (int kk = 0; kk < 3; ++kk) {
        float a2 = bqw(J, 0, kk) * vq[0];
#pragma unroll
        for (int mm = 1; mm < 4; ++mm) a2 = fmaf(bqw(J, mm, kk), vq[mm], a2);
        qu[1 + kk] = lu[1 + kk] + a2;
      }
    }
  }
  __syncwarp();  // V B, v and l_u are no longer read: K and Q_xu rows go there

  // ---- gains -----------------------------------------------------------------
  // The rare SVD fallback works in shared memory (over V B, dead here, before
  // K is written): Q at sv[0..16), its inverse at sv[16..32). Every lane of a
  // team forms the same Q and inverse, so their identical writes are benign.
  // STRAIGHT (the register tiers with room for it): the common case runs
  // straight through, the factorisation with in-range pivots (chol4_fast) and
  // the three triangular solves, and a warp with a pivot outside the normal
  // range (Q_uu not positive definite, or degenerate) repeats them for those
  // lanes through chol4 and, where that fails, the SVD inverse. Otherwise
  // (96 registers, where the longer live ranges spill) each lane branches on
  // its own factorisation. Both give the same bits.
  bool ok;
  if constexpr (STRAIGHT) {
    auto form_qs = [&](float (&Qs)[NU][NU]) {
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
    };
    Chol4 L;
    bool inr;
    {
      float Qs[NU][NU];
      form_qs(Qs);
      inr = chol4_fast(Qs, L);
    }
    auto msk = [&](int a, float v) { return (MASKED && ((tight >> a) & 1u)) ? 0.0f : v; };
    auto solve_all = [&](auto&& solve) {
      float rhs[NU], sol[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, Qxa[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) Ka[a] = -sol[a];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, Qxb[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) Kb[a] = -sol[a];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, qu[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) k[a] = -sol[a];
    };
    solve_all([&](const float (&rhs)[NU], float (&out)[NU]) { chol4_solve(L, rhs, out); });
    ok = true;
    if (__any_sync(FULL, !inr)) {
      float* sv = xc + X_K;
      if (!inr) {
        float Qs[NU][NU];
        form_qs(Qs);
        // A lane without an element (live == false) never takes the SVD path:
        // its numbers are discarded, and the warp would wait for its sweeps.
        ok = chol4(Qs, L) || !live;
        if (!ok) {
#pragma unroll
          for (int a = 0; a < NU; ++a)
#pragma unroll
            for (int b = 0; b < NU; ++b) sv[a * NU + b] = Qs[a][b];
          svd_inverse4(sv, sv + NU * NU);
        }
      }
      const bool any_fallback = __any_sync(FULL, !ok);
      if (any_fallback) __syncwarp();  // every fallback inverse of the warp is written
      if (!inr) {
        solve_all([&](const float (&rhs)[NU], float (&out)[NU]) {
          if (ok) {
            chol4_solve(L, rhs, out);
          } else {
            const float* Mi = sv + NU * NU;
#pragma unroll
            for (int a = 0; a < NU; ++a) {
              float acc = Mi[a * NU] * rhs[0];
#pragma unroll
              for (int b = 1; b < NU; ++b) acc = fmaf(Mi[a * NU + b], rhs[b], acc);
              out[a] = acc;
            }
          }
        });
      }
      if (any_fallback) __syncwarp();  // the fallback inverses are read; K goes over them
    }
  } else {
    Chol4 L;
    float* sv = xc + X_K;
    {
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
      // A lane without an element (live == false) never takes the SVD path: its
      // numbers are discarded, and the warp would wait for its sweeps.
      ok = chol4(Qs, L) || !live;
      if (!ok) {
#pragma unroll
        for (int a = 0; a < NU; ++a)
#pragma unroll
          for (int b = 0; b < NU; ++b) sv[a * NU + b] = Qs[a][b];
        svd_inverse4(sv, sv + NU * NU);
      }
    }
    const bool any_fallback = __any_sync(FULL, !ok);
    if (any_fallback) __syncwarp();  // every fallback inverse of the warp is written
    auto solve = [&](const float (&rhs)[NU], float (&out)[NU]) {
      if (ok) {
        chol4_solve(L, rhs, out);
      } else {
        const float* Mi = sv + NU * NU;
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          float acc = Mi[a * NU] * rhs[0];
#pragma unroll
          for (int b = 1; b < NU; ++b) acc = fmaf(Mi[a * NU + b], rhs[b], acc);
          out[a] = acc;
        }
      }
    };
    auto msk = [&](int a, float v) { return (MASKED && ((tight >> a) & 1u)) ? 0.0f : v; };
    {
      float rhs[NU], sol[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, Qxa[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) Ka[a] = -sol[a];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, Qxb[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) Kb[a] = -sol[a];
#pragma unroll
      for (int a = 0; a < NU; ++a) rhs[a] = msk(a, qu[a]);
      solve(rhs, sol);
#pragma unroll
      for (int a = 0; a < NU; ++a) k[a] = -sol[a];
    }
    if (any_fallback) __syncwarp();  // the fallback inverses are read; K goes over them
  }
  // K columns and Q_xu rows -> exchange (over V B, v, l_u)
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    xc[X_K + a * NX + ra] = Ka[a];
    xc[X_K + a * NX + rb] = Kb[a];
    xc[X_QXU + a * NX + ra] = Qxa[a];
    xc[X_QXU + a * NX + rb] = Qxb[a];
  }

  // ---- value update for my rows -------------------------------------------------
  // (K^T Q_uu) K + Q_xu K is formed as (K^T Q_uu + Q_xu) K: one 4-term
  // product per entry instead of two. W = K^T Q_uu + Q_xu for my rows.
  float w[NU];
  if (MASKED) {
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      float acc = Quu[a][0] * k[0];
#pragma unroll
      for (int b = 1; b < NU; ++b) acc = fmaf(Quu[a][b], k[b], acc);
      w[a] = acc + qu[a];
    }
  }
  auto wrow = [&](const float (&Kr)[NU], const float (&Qxr)[NU], float (&Wr)[NU]) {
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      float acc = Kr[0] * Quu[0][a];
#pragma unroll
      for (int b = 1; b < NU; ++b) acc = fmaf(Kr[b], Quu[b][a], acc);
      Wr[a] = acc + Qxr[a];
    }
  };
  auto vrow = [&](const float (&Kr)[NU], const float (&Qxr)[NU], const float (&Wr)[NU], float qxr) {
    if (MASKED) {
      float t2 = Kr[0] * w[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t2 = fmaf(Kr[a], w[a], t2);
      float t3 = Qxr[0] * k[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t3 = fmaf(Qxr[a], k[a], t3);
      return (qxr + t2) + t3;
    } else {
      float t1 = Wr[0] * k[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t1 = fmaf(Wr[a], k[a], t1);
      float t2 = Kr[0] * qu[0];
#pragma unroll
      for (int a = 1; a < NU; ++a) t2 = fmaf(Kr[a], qu[a], t2);
      return (qxr + t1) + t2;
    }
  };
  float Wa[NU], Wb[NU];
  wrow(Ka, Qxa, Wa);
  wrow(Kb, Qxb, Wb);
  va_ = vrow(Ka, Qxa, Wa, qxa);
  vb_ = vrow(Kb, Qxb, Wb, qxb);
  __syncwarp();  // K and Q_xu rows of the whole team are in the exchange
  // Q_xx entries of my rows are formed two columns at a time here (A^T (V A)
  // from the V A rows still in the exchange, plus l_xx), then
  // V[r][c] = (Q_xx[r][c] + W_r K_c) + K_r Q_xu[c], every sum in the order
  // of the scalar formulas (packed pairs: columns c, c + 1).
  {
    float2 wa[NU], wb[NU], ka[NU], kb[NU];
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      wa[a] = dup2(Wa[a]);
      wb[a] = dup2(Wb[a]);
      ka[a] = dup2(Ka[a]);
      kb[a] = dup2(Kb[a]);
    }
#pragma unroll
    for (int c = 0; c < NX; c += 2) {
      float2 qa = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int s = 0; s < 7; ++s) qa = fma2(c2[s], ld2(xc + X_VA + (3 + s) * NX + c), qa);
      qa = add2(Ct.pair(ra, c), fma2(c2[7], ld2(xc + X_VA + ra * NX + c), qa));
      const float2 qb = add2(Ct.pair(rb, c), fma2(cb2, ld2(xc + X_VA + pb * NX + c), ld2(xc + X_VA + rb * NX + c)));
      float2 kp[NU], qp[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        kp[a] = ld2(xc + X_K + a * NX + c);
        qp[a] = ld2(xc + X_QXU + a * NX + c);
      }
      auto entry = [&](float2 q, const float2 (&Wr)[NU], const float2 (&Kr)[NU]) {
        float2 t1 = mul2(Wr[0], kp[0]);
        t1 = fma2(Wr[1], kp[1], t1);
        t1 = fma2(Wr[2], kp[2], t1);
        t1 = fma2(Wr[3], kp[3], t1);
        float2 t2 = mul2(Kr[0], qp[0]);
        t2 = fma2(Kr[1], qp[1], t2);
        t2 = fma2(Kr[2], qp[2], t2);
        t2 = fma2(Kr[3], qp[3], t2);
        return add2(add2(q, t1), t2);
      };
      const float2 va2 = entry(qa, wa, ka), vb2 = entry(qb, wb, kb);
      Va[c] = va2.x;
      Va[c + 1] = va2.y;
      Vb[c] = vb2.x;
      Vb[c + 1] = vb2.y;
    }
  }
  after_c();  // syncs the warp: C_t and the exchange area are no longer read
  return ok;
}

// Reduce over the 5 lanes of a team (all lanes get the result); lanes 30, 31
// (mirrors of lanes 25, 26) pass base 25 and get the sixth element's sum.
__device__ __forceinline__ float team_sum(float x, int base) {
  float s = __shfl_sync(FULL, x, base);
#pragma unroll
  for (int j = 1; j < TEAM; ++j) s += __shfl_sync(FULL, x, (base + j) & 31);
  return s;
}

// Single-buffered stream of [6 x 196] C_t slabs for one warp.
struct TeamPipe {
  float* slab;      // [EPW][CBLK]
  uint64_t* bar;
  uint32_t parity;
  const CUtensorMap* tm;
  int b0;
  bool ok;

  __device__ __forceinline__ void issue(int t) {
    if (threadIdx.x == 0) {
      fence_proxy_async();
      mbar_expect_tx(bar, TSLAB_BYTES);
      tma_load_3d(slab, tm, bar, 0, t, b0);
    }
  }
  // Runs body(t, next) over t (reverse if rev). body must call next() exactly
  // once, after its last read of the slab; next() syncs the warp and starts
  // the copy of the following step. With dense == false no copy is made:
  // fill(t) runs before body(t) instead (it may write the slab) and the warp
  // syncs after it. Returns false on a (bounded) wait timeout.
  template <class Fill, class F>
  __device__ __forceinline__ bool run(int T, bool rev, bool dense, Fill&& fill, F&& body) {
    if (dense) issue(rev ? T - 1 : 0);
    for (int s = 0; s < T; ++s) {
      const int t = rev ? T - 1 - s : s;
      if (dense) {
        const bool got = mbar_wait(bar, parity);
        if (!__all_sync(FULL, got)) {
          mbar_wait(bar, parity);  // give the copy in flight one more bounded wait
          ok = false;
          return false;
        }
        parity ^= 1u;
      } else {
        fill(t);
        __syncwarp();
      }
      bool called = false;
      auto next = [&]() {
        __syncwarp();
        if (dense && s + 1 < T) issue(rev ? t - 1 : t + 1);
        called = true;
      };
      body(t, next);
      if (!called) next();
    }
    return true;
  }
  template <class F>
  __device__ __forceinline__ bool run(int T, bool rev, F&& body) {
    return run(T, rev, true, [](int) {}, body);
  }
};

}  // namespace ilqr
