// ilqr_pnqp.cuh -- PNQP-4: the 4-dimensional box-constrained QP
//   min 1/2 x^T H x + q^T x  subject to  lower <= x <= upper
// by the projected-Newton method of mpc.pytorch's pnqp
// (acmpc_public-master/mpc.pytorch/mpc/pnqp.py:5-84) with the reference
// extension's per-problem settings (differentialMPCPerformance/cpp/
// pnqp_kernel.cuh:91-208): at most 10 Newton steps, at most 10 Armijo trials
// (gamma 0.1, step decay 0.1), a 1e-11 ridge on the reduced Hessian, stop when
// ||dx|| < 1e-4, a bound counts as active within 1e-8. A zero starting point
// starts from the unconstrained solution. Used by the batched entry point
// (ilqr_pnqp.cu) and by the FastMPC-numerics Riccati pass (ilqr_fastmpc.cu).
#pragma once

namespace ilqr {
namespace pnqp {

// A x = b for one 4x4 system by Gaussian elimination with partial pivoting;
// a pivot of magnitude below 1e-10 is replaced by +-1e-10. A and b are
// overwritten; the solution is returned in b.
__device__ __forceinline__ void solve4_pivot(float (&A)[4][4], float (&b)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int r = k;
    float best = fabsf(A[k][k]);
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      const float v = fabsf(A[i][k]);
      if (v > best) {
        best = v;
        r = i;
      }
    }
    // row swap with compile-time indices (r is a runtime value; indexing by
    // it would move A to local memory)
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      if (i == r) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float tmp = A[k][j];
          A[k][j] = A[i][j];
          A[i][j] = tmp;
        }
        const float tb = b[k];
        b[k] = b[i];
        b[i] = tb;
      }
    }
    float piv = A[k][k];
    if (fabsf(piv) < 1e-10f) piv = piv < 0.0f ? -1e-10f : 1e-10f;
#pragma unroll
    for (int i = k + 1; i < 4; ++i) {
      const float f = A[i][k] / piv;
#pragma unroll
      for (int j = k + 1; j < 4; ++j) A[i][j] = A[i][j] - f * A[k][j];
      b[i] = b[i] - f * b[k];
      A[i][k] = 0.0f;
    }
  }
#pragma unroll
  for (int i = 3; i >= 0; --i) {
    float s = b[i];
#pragma unroll
    for (int j = i + 1; j < 4; ++j) s = s - A[i][j] * b[j];
    b[i] = s / A[i][i];
  }
}

__device__ __forceinline__ void hx_plus_q(const float (&H)[4][4], const float (&q)[4], const float (&x)[4],
                                          float (&g)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float s = H[i][0] * x[0];
#pragma unroll
    for (int j = 1; j < 4; ++j) s = fmaf(H[i][j], x[j], s);
    g[i] = s + q[i];
  }
}

__device__ __forceinline__ float objective(const float (&H)[4][4], const float (&q)[4], const float (&x)[4]) {
  float quad = 0.0f, lin = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float hx = H[i][0] * x[0];
#pragma unroll
    for (int j = 1; j < 4; ++j) hx = fmaf(H[i][j], x[j], hx);
    quad = fmaf(x[i], hx, quad);
    lin = fmaf(q[i], x[i], lin);
  }
  return 0.5f * quad + lin;
}

// Solves one problem: x holds the starting point on entry and the optimum on
// return; fr[i] is 1 for coordinates not held at a bound by the final
// gradient, else 0.
__device__ __forceinline__ void pnqp4(const float (&H)[4][4], const float (&q)[4], const float (&lo)[4],
                                      const float (&hi)[4], float (&x)[4], float (&fr)[4]) {
  constexpr float EPS_BOUND = 1e-8f, GAMMA = 0.1f, DECAY = 0.1f, RIDGE = 1e-11f, TOL2 = 1e-8f;
  if (x[0] == 0.0f && x[1] == 0.0f && x[2] == 0.0f && x[3] == 0.0f) {
    float A[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) A[i][j] = H[i][j];
      x[i] = -q[i];
    }
    solve4_pivot(A, x);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = fminf(fmaxf(x[i], lo[i]), hi[i]);

  for (int it = 0; it < 10; ++it) {
    float g[4];
    hx_plus_q(H, q, x, g);
    float fr[4], A[4][4], dx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool held = (x[i] <= lo[i] + EPS_BOUND && g[i] > 0.0f) || (x[i] >= hi[i] - EPS_BOUND && g[i] < 0.0f);
      fr[i] = held ? 0.0f : 1.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) A[i][j] = H[i][j] * fr[i] * fr[j];
      A[i][i] += RIDGE;
      dx[i] = -g[i] * fr[i];
    }
    solve4_pivot(A, dx);
    float n2 = dx[0] * dx[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) n2 = fmaf(dx[i], dx[i], n2);
    if (n2 < TOL2) break;
    const float ox = objective(H, q, x);
    float alpha = 1.0f, mx[4];
    for (int ls = 0; ls < 10; ++ls) {
#pragma unroll
      for (int i = 0; i < 4; ++i) mx[i] = fminf(fmaxf(fmaf(alpha, dx[i], x[i]), lo[i]), hi[i]);
      const float om = objective(H, q, mx);
      float den = g[0] * (x[0] - mx[0]);
#pragma unroll
      for (int i = 1; i < 4; ++i) den = fmaf(g[i], x[i] - mx[i], den);
      const float armijo = (ox - om) / (fabsf(den) > 1e-12f ? den : 1e-12f);
      if (armijo > GAMMA) break;
      alpha *= DECAY;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = mx[i];
  }
  float g[4];
  hx_plus_q(H, q, x, g);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool held = (x[i] <= lo[i] + EPS_BOUND && g[i] > 0.0f) || (x[i] >= hi[i] - EPS_BOUND && g[i] < 0.0f);
    fr[i] = held ? 0.0f : 1.0f;
  }
}

}  // namespace pnqp
}  // namespace ilqr
