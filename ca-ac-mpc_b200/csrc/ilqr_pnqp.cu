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
#include "ilqr_pnqp.cuh"

namespace ilqr {

namespace {

__global__ void __launch_bounds__(128) pnqp4_batch_kernel(const float* __restrict__ Hg, const float* __restrict__ qg,
                                                         const float* __restrict__ lg, const float* __restrict__ ug,
                                                         const float* __restrict__ xg, int64_t n,
                                                         float* __restrict__ x_out, float* __restrict__ free_out) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  float H[4][4], q[4], lo[4], hi[4], x[4], fr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) H[i][j] = __ldg(Hg + b * 16 + i * 4 + j);
    q[i] = __ldg(qg + b * 4 + i);
    lo[i] = __ldg(lg + b * 4 + i);
    hi[i] = __ldg(ug + b * 4 + i);
    x[i] = xg != nullptr ? __ldg(xg + b * 4 + i) : 0.0f;
  }
  pnqp::pnqp4(H, q, lo, hi, x, fr);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x_out[b * 4 + i] = x[i];
    free_out[b * 4 + i] = fr[i];
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
