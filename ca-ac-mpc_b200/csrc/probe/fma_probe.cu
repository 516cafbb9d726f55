// fma_probe.cu -- FP32 FMA throughput probe (measurement only; built into
// libilqr_probe.so, not part of the solver library). Each thread runs
// `iters` rounds of 8 independent FMA chains; the caller times the launch.
#include <cuda_runtime.h>
#include <stdint.h>

__global__ void fma_probe_kernel(float* out, int iters, float a, float b) {
  float r0 = threadIdx.x, r1 = r0 + 1, r2 = r0 + 2, r3 = r0 + 3, r4 = r0 + 4, r5 = r0 + 5, r6 = r0 + 6,
        r7 = r0 + 7;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      r0 = fmaf(r0, a, b); r1 = fmaf(r1, a, b); r2 = fmaf(r2, a, b); r3 = fmaf(r3, a, b);
      r4 = fmaf(r4, a, b); r5 = fmaf(r5, a, b); r6 = fmaf(r6, a, b); r7 = fmaf(r7, a, b);
    }
  }
  const float s = ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7));
  if (s == 1234.5f) out[blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the chains live
}

extern "C" int ilqr_probe_fma(float* out, int blocks, int threads, int iters, void* stream) {
  fma_probe_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(out, iters, 0.999999f, 1e-7f);
  return (int)cudaGetLastError();
}

// FLOPs of one launch: blocks * threads * iters * 16 * 8 FMAs * 2.
extern "C" double ilqr_probe_fma_flops(int blocks, int threads, int iters) {
  return (double)blocks * threads * iters * 16.0 * 8.0 * 2.0;
}
