// ilqr_compat.cu -- kernels behind the reference extension's secondary entry
// points: the model step, Jacobian materialisation (A_lin, B_lin of
// drone_ilqr_solve's return tuple), and the explicit-A/B adjoint Riccati and
// gradient assembly (drone_backward_pass_batched, drone_implicit_diff_assembly)
// for callers that hold their own linearisation. The fused solve/backward
// kernels do not use these.
#include "ilqr_device.cuh"
#include "ilqr_kernels.h"

namespace ilqr {

namespace {

__global__ void dynamics_kernel(const float* __restrict__ x, const float* __restrict__ u, int64_t n, float dt,
                                float* __restrict__ xn) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xs[NX], us[NU], out[NX];
#pragma unroll
  for (int k = 0; k < NX; ++k) xs[k] = x[i * NX + k];
#pragma unroll
  for (int k = 0; k < NU; ++k) us[k] = u[i * NU + k];
  drone_step(xs, us, dt, out);
#pragma unroll
  for (int k = 0; k < NX; ++k) xn[i * NX + k] = out[k];
}

// A = I + dt J_x, B = dt J_u at (X[b,t], U[b,t]), written dense.
__global__ void linearize_kernel(const float* __restrict__ X, const float* __restrict__ U, int64_t B, int T,
                                 float dt, float* __restrict__ A, float* __restrict__ Bm) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int64_t b = i / T, t = i % T;
  float xs[NX], us[NU];
#pragma unroll
  for (int k = 0; k < NX; ++k) xs[k] = X[(b * (T + 1) + t) * NX + k];
#pragma unroll
  for (int k = 0; k < NU; ++k) us[k] = U[i * NU + k];
  const Jac J = drone_jac(xs, us, dt);
  float* Ai = A + i * NX * NX;
  float* Bi = Bm + i * NX * NU;
  for (int r = 0; r < NX; ++r)
    for (int c = 0; c < NX; ++c) {
      float val = (r == c) ? 1.0f : 0.0f;
      if (r < 3 && c == 7 + r) val = J.dt;
      if (r >= 3 && r < 7 && c >= 3 && c < 7) val = aqq(J, r - 3, c - 3);
      if (r >= 7 && c >= 3 && c < 7) val = avq(J, r - 7, c - 3);
      Ai[r * NX + c] = val;
    }
  for (int r = 0; r < NX; ++r)
    for (int a = 0; a < NU; ++a) {
      float val = 0.0f;
      if (r >= 3 && r < 7 && a >= 1) val = bqw(J, r - 3, a - 1);
      if (r >= 7 && a == 0) val = bvf(J, r - 7);
      Bi[r * NU + a] = val;
    }
}

// Masked adjoint Riccati on caller-supplied dense A, B (_zero_constrained_lqr,
// controller.py:1035-1110): V_A = V A, V_B = V B, Q_xx = l_xx + A^T V_A, ...
// Per-thread matrices live in local memory; this is a compatibility path.
__global__ void adjoint_lqr_kernel(const float* __restrict__ A, const float* __restrict__ Bm,
                                   const float* __restrict__ l_xx, const float* __restrict__ l_uu,
                                   const float* __restrict__ l_xu, const float* __restrict__ l_x,
                                   const float* __restrict__ l_u, const float* __restrict__ l_xxN,
                                   const float* __restrict__ l_xN, const uint8_t* __restrict__ tight, int64_t B,
                                   int T, float reg, float* __restrict__ Kout, float* __restrict__ kout,
                                   float* __restrict__ v0) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float V[NX][NX], v[NX];
  for (int i = 0; i < NX; ++i) {
    v[i] = l_xN[b * NX + i];
    for (int j = 0; j < NX; ++j) V[i][j] = l_xxN[b * NX * NX + i * NX + j];
  }
  for (int t = T - 1; t >= 0; --t) {
    const int64_t bt = b * T + t;
    const float* At = A + bt * NX * NX;
    const float* Bt = Bm + bt * NX * NU;
    float VA[NX][NX], VB[NX][NU];
    for (int i = 0; i < NX; ++i) {
      for (int j = 0; j < NX; ++j) {
        float acc = V[i][0] * At[j];
        for (int k = 1; k < NX; ++k) acc = fmaf(V[i][k], At[k * NX + j], acc);
        VA[i][j] = acc;
      }
      for (int a = 0; a < NU; ++a) {
        float acc = V[i][0] * Bt[a];
        for (int k = 1; k < NX; ++k) acc = fmaf(V[i][k], Bt[k * NU + a], acc);
        VB[i][a] = acc;
      }
    }
    float Qxx[NX][NX], Qxu[NX][NU], Quu[NU][NU], qx[NX], qu[NU];
    for (int i = 0; i < NX; ++i) {
      for (int j = 0; j < NX; ++j) {
        float acc = At[i] * VA[0][j];
        for (int k = 1; k < NX; ++k) acc = fmaf(At[k * NX + i], VA[k][j], acc);
        Qxx[i][j] = l_xx[bt * NX * NX + i * NX + j] + acc;
      }
      for (int a = 0; a < NU; ++a) {
        float acc = At[i] * VB[0][a];
        for (int k = 1; k < NX; ++k) acc = fmaf(At[k * NX + i], VB[k][a], acc);
        Qxu[i][a] = l_xu[bt * NX * NU + i * NU + a] + acc;
      }
      float acc = At[i] * v[0];
      for (int k = 1; k < NX; ++k) acc = fmaf(At[k * NX + i], v[k], acc);
      qx[i] = l_x[bt * NX + i] + acc;
    }
    for (int a = 0; a < NU; ++a) {
      for (int c = 0; c < NU; ++c) {
        float acc = Bt[a] * VB[0][c];
        for (int k = 1; k < NX; ++k) acc = fmaf(Bt[k * NU + a], VB[k][c], acc);
        Quu[a][c] = (l_uu[bt * NU * NU + a * NU + c] + acc) + (a == c ? reg : 0.0f);
      }
      float acc = Bt[a] * v[0];
      for (int k = 1; k < NX; ++k) acc = fmaf(Bt[k * NU + a], v[k], acc);
      qu[a] = l_u[bt * NU + a] + acc;
    }
    uint32_t m = 0;
    if (tight != nullptr)
      for (int a = 0; a < NU; ++a) m |= (tight[bt * NU + a] != 0 ? 1u : 0u) << a;
    float Qs[NU][NU];
    for (int a = 0; a < NU; ++a)
      for (int c = 0; c < NU; ++c) {
        const bool ta = (m >> a) & 1u, tc = (m >> c) & 1u;
        float val = (ta || tc) ? 0.0f : Quu[a][c];
        if (a == c && ta) val = val + 1.0f;
        Qs[a][c] = val + (a == c ? 1e-8f * reg : 0.0f);
      }
    Chol4 L;
    float Mi[NU][NU];
    const bool ok = chol4(Qs, L);
    if (!ok) svd_inverse4(&Qs[0][0], &Mi[0][0]);
    float K[NU][NX], k[NU];
    for (int j = 0; j <= NX; ++j) {
      float rhs[NU], sol[NU];
      for (int a = 0; a < NU; ++a) {
        const float val = (j < NX) ? Qxu[j][a] : qu[a];
        rhs[a] = ((m >> a) & 1u) ? 0.0f : val;
      }
      if (ok) {
        chol4_solve(L, rhs, sol);
      } else {
        for (int a = 0; a < NU; ++a) {
          float acc = Mi[a][0] * rhs[0];
          for (int c = 1; c < NU; ++c) acc = fmaf(Mi[a][c], rhs[c], acc);
          sol[a] = acc;
        }
      }
      for (int a = 0; a < NU; ++a) {
        if (j < NX) K[a][j] = -sol[a]; else k[a] = -sol[a];
      }
    }
    for (int a = 0; a < NU; ++a) {
      for (int j = 0; j < NX; ++j) Kout[(bt * NU + a) * NX + j] = K[a][j];
      kout[bt * NU + a] = k[a];
    }
    // V = Q_xx + K^T (Q_uu K) + K^T Q_ux + Q_xu K; v = q_x + K^T (Q_uu k + q_u) + Q_xu k
    float W[NU][NX], w[NU];
    for (int a = 0; a < NU; ++a) {
      for (int j = 0; j < NX; ++j) {
        float acc = Quu[a][0] * K[0][j];
        for (int c = 1; c < NU; ++c) acc = fmaf(Quu[a][c], K[c][j], acc);
        W[a][j] = acc;
      }
      float acc = Quu[a][0] * k[0];
      for (int c = 1; c < NU; ++c) acc = fmaf(Quu[a][c], k[c], acc);
      w[a] = acc + qu[a];
    }
    for (int i = 0; i < NX; ++i) {
      for (int j = 0; j < NX; ++j) {
        float t1 = K[0][i] * W[0][j], t2 = K[0][i] * Qxu[j][0], t3 = Qxu[i][0] * K[0][j];
        for (int a = 1; a < NU; ++a) {
          t1 = fmaf(K[a][i], W[a][j], t1);
          t2 = fmaf(K[a][i], Qxu[j][a], t2);
          t3 = fmaf(Qxu[i][a], K[a][j], t3);
        }
        V[i][j] = ((Qxx[i][j] + t1) + t2) + t3;
      }
      float t2 = K[0][i] * w[0], t3 = Qxu[i][0] * k[0];
      for (int a = 1; a < NU; ++a) {
        t2 = fmaf(K[a][i], w[a], t2);
        t3 = fmaf(Qxu[i][a], k[a], t3);
      }
      v[i] = (qx[i] + t2) + t3;
    }
  }
  for (int i = 0; i < NX; ++i) v0[b * NX + i] = v[i];
}

// Sweep and gradients from (K, k, v0) with dense A, B (ILQRSolve.backward,
// controller.py:84-125).
__global__ void assembly_kernel(const float* __restrict__ K, const float* __restrict__ k,
                                const float* __restrict__ v0, const float* __restrict__ A,
                                const float* __restrict__ Bm, const float* __restrict__ X,
                                const float* __restrict__ U, const float* __restrict__ x_ref, int64_t B, int T,
                                float* gC, float* gc, float* gx0, float* gxr, float* gur, float* gCf, float* gcf) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (gx0 != nullptr)
    for (int i = 0; i < NX; ++i) gx0[b * NX + i] = -v0[b * NX + i];
  float dx[NX];
  for (int i = 0; i < NX; ++i) dx[i] = 0.0f;
  for (int t = 0; t < T; ++t) {
    const int64_t bt = b * T + t;
    float z[NT], dtau[NT], du[NU];
    for (int i = 0; i < NX; ++i) z[i] = X[(b * (T + 1) + t) * NX + i];
    for (int a = 0; a < NU; ++a) z[NX + a] = U[bt * NU + a];
    for (int a = 0; a < NU; ++a) {
      float acc = K[(bt * NU + a) * NX] * dx[0];
      for (int j = 1; j < NX; ++j) acc = fmaf(K[(bt * NU + a) * NX + j], dx[j], acc);
      du[a] = acc + k[bt * NU + a];
    }
    for (int i = 0; i < NX; ++i) dtau[i] = dx[i];
    for (int a = 0; a < NU; ++a) dtau[NX + a] = du[a];
    if (gC != nullptr)
      for (int i = 0; i < NT; ++i)
        for (int j = 0; j < NT; ++j) gC[bt * CBLK + i * NT + j] = -0.5f * (dtau[i] * z[j] + z[i] * dtau[j]);
    if (gc != nullptr)
      for (int i = 0; i < NT; ++i) gc[bt * NT + i] = -dtau[i];
    if (gxr != nullptr)
      for (int i = 0; i < NX; ++i) gxr[(b * (T + 1) + t) * NX + i] = dx[i];
    if (gur != nullptr)
      for (int a = 0; a < NU; ++a) gur[bt * NU + a] = du[a];
    const float* At = A + bt * NX * NX;
    const float* Bt = Bm + bt * NX * NU;
    float nd[NX];
    for (int i = 0; i < NX; ++i) {
      float a1 = At[i * NX] * dx[0];
      for (int j = 1; j < NX; ++j) a1 = fmaf(At[i * NX + j], dx[j], a1);
      float a2 = Bt[i * NU] * du[0];
      for (int a = 1; a < NU; ++a) a2 = fmaf(Bt[i * NU + a], du[a], a2);
      nd[i] = a1 + a2;
    }
    for (int i = 0; i < NX; ++i) dx[i] = nd[i];
  }
  if (gxr != nullptr)
    for (int i = 0; i < NX; ++i) gxr[(b * (T + 1) + T) * NX + i] = 0.0f;
  float e[NX];
  for (int i = 0; i < NX; ++i)
    e[i] = X[(b * (T + 1) + T) * NX + i] - (x_ref != nullptr ? x_ref[(b * (T + 1) + T) * NX + i] : 0.0f);
  if (gCf != nullptr)
    for (int i = 0; i < NT; ++i)
      for (int j = 0; j < NT; ++j)
        gCf[b * CBLK + i * NT + j] = (i < NX && j < NX) ? -0.5f * (dx[i] * e[j] + e[i] * dx[j]) : 0.0f;
  if (gcf != nullptr)
    for (int i = 0; i < NT; ++i) gcf[b * NT + i] = i < NX ? -dx[i] : 0.0f;
}

unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

cudaError_t launch_dynamics(const float* x, const float* u, int64_t n, float dt, float* xn, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  dynamics_kernel<<<blocks_for(n, 128), 128, 0, s>>>(x, u, n, dt, xn);
  return cudaGetLastError();
}

cudaError_t launch_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A, float* Bm,
                             cudaStream_t s) {
  if (B * T == 0) return cudaSuccess;
  linearize_kernel<<<blocks_for(B * T, 128), 128, 0, s>>>(X, U, B, T, dt, A, Bm);
  return cudaGetLastError();
}

cudaError_t launch_adjoint_lqr(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                               const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                               const float* l_xN, const uint8_t* tight, int64_t B, int T, float reg, float* K,
                               float* k, float* v0, cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  adjoint_lqr_kernel<<<blocks_for(B, 64), 64, 0, s>>>(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN, tight, B,
                                                       T, reg, K, k, v0);
  return cudaGetLastError();
}

cudaError_t launch_assembly(const float* K, const float* k, const float* v0, const float* A, const float* Bm,
                            const float* X, const float* U, const float* x_ref, const float* u_ref, int64_t B,
                            int T, float* gC, float* gc, float* gx0, float* gxr, float* gur, float* gCf,
                            float* gcf, cudaStream_t s) {
  (void)u_ref;
  if (B == 0) return cudaSuccess;
  assembly_kernel<<<blocks_for(B, 64), 64, 0, s>>>(K, k, v0, A, Bm, X, U, x_ref, B, T, gC, gc, gx0, gxr, gur, gCf,
                                                    gcf);
  return cudaGetLastError();
}

}  // namespace ilqr
