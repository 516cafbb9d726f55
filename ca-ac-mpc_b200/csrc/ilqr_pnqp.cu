// ilqr_pnqp.cu -- batched 4-dimensional box-constrained QP (drone_pnqp4_batch).
//
// min 1/2 x^T H x + q^T x subject to lower <= x <= upper, one thread per
// problem: the projected-Newton method of mpc.pytorch's pnqp
// (acmpc_public-master/mpc.pytorch/mpc/pnqp.py:5-84) per problem, with the
// reference extension's per-problem settings (differentialMPCPerformance/cpp/
// pnqp_kernel.cuh:91-208): at most 10 Newton steps, at most 10 Armijo trials
// (gamma 0.1, step decay 0.1), a 1e-11 ridge on the reduced Hessian, stop when
// ||dx|| < 1e-4, a bound counts as active within 1e-8. A zero (or absent)
// starting point starts from the unconstrained solution. The free mask is
// 1 for coordinates not held at a bound by the final gradient.
#include "ilqr_kernels.h"
#include "ilqr_device.cuh"

namespace ilqr {

namespace {

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
    if (r != k) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float tmp = A[k][j];
        A[k][j] = A[r][j];
        A[r][j] = tmp;
      }
      const float tb = b[k];
      b[k] = b[r];
      b[r] = tb;
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

__global__ void __launch_bounds__(128) pnqp4_batch_kernel(const float* __restrict__ Hg, const float* __restrict__ qg,
                                                         const float* __restrict__ lg, const float* __restrict__ ug,
                                                         const float* __restrict__ xg, int64_t n,
                                                         float* __restrict__ x_out, float* __restrict__ free_out) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  constexpr float EPS_BOUND = 1e-8f, GAMMA = 0.1f, DECAY = 0.1f, RIDGE = 1e-11f, TOL2 = 1e-8f;
  float H[4][4], q[4], lo[4], hi[4], x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) H[i][j] = __ldg(Hg + b * 16 + i * 4 + j);
    q[i] = __ldg(qg + b * 4 + i);
    lo[i] = __ldg(lg + b * 4 + i);
    hi[i] = __ldg(ug + b * 4 + i);
    x[i] = xg != nullptr ? __ldg(xg + b * 4 + i) : 0.0f;
  }
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
    x_out[b * 4 + i] = x[i];
    free_out[b * 4 + i] = held ? 0.0f : 1.0f;
  }
}

}  // namespace

cudaError_t launch_pnqp4_batch(const float* H, const float* q, const float* lower, const float* upper,
                               const float* x_init, int64_t n, float* x_out, float* free_mask, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + 127) / 128);
  pnqp4_batch_kernel<<<grid, 128, 0, stream>>>(H, q, lower, upper, x_init, n, x_out, free_mask);
  return cudaGetLastError();
}

}  // namespace ilqr
