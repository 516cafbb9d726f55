// ilqr_backward.cu -- fused implicit-differentiation backward pass.
//
// One CTA = one warp = 32 batch elements, one thread per element. Two passes
// over the horizon:
//   1. reverse: masked adjoint Riccati (controller.py:1035-1110) with A_t, B_t
//      recomputed from (X_t, U_t) and l_xx, l_xu, l_uu read from the TMA-staged
//      C_t slab; gains (K_t, k_t) go to an element-interleaved workspace.
//   2. forward: dU = K dX + k, dX+ = A dX + B dU (controller.py:1121-1129) and
//      the gradients of ILQRSolve.backward (controller.py:84-125). grad_C[b, t]
//      (784 B per element and step) is written into a [32 x 196] shared-memory
//      slab and stored with one TMA bulk tensor store per step.
#include "ilqr_device.cuh"
#include "ilqr_kernels.h"

namespace ilqr {

namespace {

__global__ void __launch_bounds__(WARP) backward_kernel(const __grid_constant__ CUtensorMap tmC,
                                                        const __grid_constant__ CUtensorMap tmG,
                                                        const BackwardParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* cbuf = reinterpret_cast<float*>(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * SLAB_BYTES);
  const int lane = threadIdx.x;
  const int64_t b0 = (int64_t)blockIdx.x * WARP;
  const int64_t b = b0 + lane;
  const bool valid = b < p.B;
  const int T = p.T;
  const int64_t S = p.S;
  const float dt = p.dt;
  float* Kw = p.ws + b;
  float* kw = p.ws + (int64_t)T * NU * NX * S + b;
  auto Kat = [&](int t, int a, int j) -> float& { return Kw[(int64_t)(t * NU * NX + a * NX + j) * S]; };
  auto kat = [&](int t, int a) -> float& { return kw[(int64_t)(t * NU + a) * S]; };
  auto ld = [&](const float* q, int64_t i) { return valid ? __ldg(q + i) : 0.0f; };

  if (lane == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncwarp();
  CPipe pipe{cbuf, bar, 0u, &tmC, (int)b0};

  const float* Xb = p.X + b * (int64_t)(T + 1) * NX;
  const float* Ub = p.U + b * (int64_t)T * NU;
  const float* gXb = p.gX + b * (int64_t)(T + 1) * NX;
  const float* gUb = p.gU + b * (int64_t)T * NU;
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;

  // ---- 1. masked adjoint Riccati, V_T = C_f[:nx,:nx], v_T = -dL/dX_T --------
  float V[NX][NX], v[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) {
    v[i] = -ld(gXb, T * NX + i);
#pragma unroll
    for (int j = 0; j < NX; ++j) V[i][j] = Cf ? __ldg(Cf + i * NT + j) : 0.0f;
  }
  bool ok = pipe.run(T, true, [&](int t, const float* Crow) {
    float xb[NX], ub[NU], lx[NX], lu[NU];
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      xb[i] = ld(Xb, t * NX + i);
      lx[i] = -ld(gXb, t * NX + i);
    }
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      ub[a] = ld(Ub, t * NU + a);
      lu[a] = -ld(gUb, t * NU + a);
    }
    uint32_t tight = 0;
    if (p.tight != nullptr && valid) {
#pragma unroll
      for (int a = 0; a < NU; ++a) tight |= (p.tight[(b * T + t) * NU + a] != 0 ? 1u : 0u) << a;
    }
    const Jac J = drone_jac(xb, ub, dt);
    float K[NU][NX], k[NU];
    riccati_step<true>(V, v, J, Crow, lx, lu, p.reg, tight, K, k);
#pragma unroll
    for (int a = 0; a < NU; ++a) {
#pragma unroll
      for (int j = 0; j < NX; ++j) Kat(t, a, j) = K[a][j];
      kat(t, a) = k[a];
    }
  });
  if (!ok) return;  // bounded wait gave up; outputs are left untouched
  if (valid && p.g_x0 != nullptr) {
#pragma unroll
    for (int i = 0; i < NX; ++i) p.g_x0[b * NX + i] = -v[i];
  }

  // ---- 2. tangent sweep and gradient assembly -------------------------------
  float dx[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) dx[i] = 0.0f;
  for (int t = 0; t < T; ++t) {
    float z[NT], du[NU];
#pragma unroll
    for (int i = 0; i < NX; ++i) z[i] = ld(Xb, t * NX + i);
#pragma unroll
    for (int a = 0; a < NU; ++a) z[NX + a] = ld(Ub, t * NU + a);
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      float acc = Kat(t, a, 0) * dx[0];
#pragma unroll
      for (int j = 1; j < NX; ++j) acc = fmaf(Kat(t, a, j), dx[j], acc);
      du[a] = acc + kat(t, a);
    }
    float dtau[NT];
#pragma unroll
    for (int i = 0; i < NX; ++i) dtau[i] = dx[i];
#pragma unroll
    for (int a = 0; a < NU; ++a) dtau[NX + a] = du[a];
    if (p.write_gC) {
      const int slot = t & 1;
      if (t >= 2) {
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
      }
      float4* row = reinterpret_cast<float4*>(cbuf + slot * CSLAB + lane * CBLK);
#pragma unroll
      for (int q = 0; q < CBLK / 4; ++q) {
        float g[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int e = 4 * q + m, i = e / NT, j = e % NT;
          g[m] = -0.5f * (dtau[i] * z[j] + z[i] * dtau[j]);
        }
        row[q] = make_float4(g[0], g[1], g[2], g[3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tmG, cbuf + slot * CSLAB, 0, t, (int)b0);
        bulk_commit();
      }
    }
    if (valid) {
      if (p.g_c != nullptr) {
#pragma unroll
        for (int i = 0; i < NT; ++i) p.g_c[(b * T + t) * NT + i] = -dtau[i];
      }
      if (p.g_xref != nullptr) {
#pragma unroll
        for (int i = 0; i < NX; ++i) p.g_xref[(b * (T + 1) + t) * NX + i] = dx[i];
      }
      if (p.g_uref != nullptr) {
#pragma unroll
        for (int a = 0; a < NU; ++a) p.g_uref[(b * T + t) * NU + a] = du[a];
      }
    }
    float xs[NX], us[NU];
#pragma unroll
    for (int i = 0; i < NX; ++i) xs[i] = z[i];
#pragma unroll
    for (int a = 0; a < NU; ++a) us[a] = z[NX + a];
    const Jac J = drone_jac(xs, us, dt);
    float nd[NX];
    jac_apply(J, dx, du, nd);
#pragma unroll
    for (int i = 0; i < NX; ++i) dx[i] = nd[i];
  }
  if (p.write_gC && lane == 0) bulk_wait<0>();
  __syncwarp();
  if (!valid) return;
  if (p.g_xref != nullptr) {
#pragma unroll
    for (int i = 0; i < NX; ++i) p.g_xref[(b * (T + 1) + T) * NX + i] = 0.0f;
  }
  if (p.g_Cf != nullptr || p.g_cf != nullptr) {
    float e[NX];
#pragma unroll
    for (int i = 0; i < NX; ++i)
      e[i] = ld(Xb, T * NX + i) - (p.x_ref != nullptr ? __ldg(p.x_ref + (b * (T + 1) + T) * NX + i) : 0.0f);
    if (p.g_Cf != nullptr) {
      for (int i = 0; i < NT; ++i)
        for (int j = 0; j < NT; ++j)
          p.g_Cf[b * CBLK + i * NT + j] = (i < NX && j < NX) ? -0.5f * (dx[i] * e[j] + e[i] * dx[j]) : 0.0f;
    }
    if (p.g_cf != nullptr) {
      for (int i = 0; i < NT; ++i) p.g_cf[b * NT + i] = i < NX ? -dx[i] : 0.0f;
    }
  }
}

}  // namespace

size_t backward_smem_bytes() { return 2 * SLAB_BYTES + 2 * sizeof(uint64_t); }

cudaError_t launch_backward(const CUtensorMap& tmC, const CUtensorMap& tmG, const BackwardParams& p,
                            cudaStream_t stream) {
  const size_t smem = backward_smem_bytes();
  const unsigned grid = (unsigned)((p.B + WARP - 1) / WARP);
  cudaError_t e = cudaFuncSetAttribute(backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  backward_kernel<<<grid, WARP, smem, stream>>>(tmC, tmG, p);
  return cudaGetLastError();
}

}  // namespace ilqr
