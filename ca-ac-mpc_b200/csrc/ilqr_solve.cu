// ilqr_solve.cu -- fused batched iLQR forward solve (all iterations, one launch).
//
// Mapping: one CTA = one warp = 32 batch elements, one thread per element.
// Per-element trajectories (nominal X, U) and gains (K, k) live in a
// caller-provided workspace in an element-interleaved layout
// (field f of element b at ws[f * S + b], S = B rounded up to 32), so every
// workspace access of a warp is one coalesced 128-byte transaction. The dense
// cost blocks C[b, t] (784 B per element and step) are staged into shared
// memory by TMA, one [32 x 196] slab per time step, double-buffered, so the
// copy of step t+-1 overlaps the math of step t.
//
// Algorithm: DifferentiableMPCController.solve_step (controller.py:303-435)
// with per-element freezing (see oracle notes): an element stops at its first
// non-improving iteration, which leaves X, U identical to the reference's
// global loop.
#include "ilqr_device.cuh"
#include "ilqr_kernels.h"

namespace ilqr {

namespace {

struct Ws {
  float* Xn;  // [(T+1)*10] fields
  float* Un;  // [T*4]
  float* K;   // [T*40]
  float* k;   // [T*4]
  int64_t S;
  __device__ __forceinline__ float& x(int t, int i) const { return Xn[(int64_t)(t * NX + i) * S]; }
  __device__ __forceinline__ float& u(int t, int a) const { return Un[(int64_t)(t * NU + a) * S]; }
  __device__ __forceinline__ float& K_(int t, int a, int j) const { return K[(int64_t)(t * NU * NX + a * NX + j) * S]; }
  __device__ __forceinline__ float& k_(int t, int a) const { return k[(int64_t)(t * NU + a) * S]; }
};

__device__ __forceinline__ float ldg_or0(const float* p, bool ok) { return ok ? __ldg(p) : 0.0f; }

// q += tau^T C tau, one 14x14 block read row by row from shared memory.
template <int NA>
__device__ __forceinline__ void quad_accum(const float* __restrict__ Crow, const float (&tau)[NA][NT],
                                           float (&sq)[NA]) {
  float q[NA];
#pragma unroll
  for (int a = 0; a < NA; ++a) q[a] = 0.0f;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    float c[NT];
    const float2* r2 = reinterpret_cast<const float2*>(Crow + i * NT);
#pragma unroll
    for (int j = 0; j < NT / 2; ++j) {
      const float2 v = r2[j];
      c[2 * j] = v.x;
      c[2 * j + 1] = v.y;
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      float r = c[0] * tau[a][0];
#pragma unroll
      for (int j = 1; j < NT; ++j) r = fmaf(c[j], tau[a][j], r);
      q[a] = fmaf(tau[a][i], r, q[a]);
    }
  }
#pragma unroll
  for (int a = 0; a < NA; ++a) sq[a] += q[a];
}

template <int NA>
__device__ __forceinline__ void lin_accum(const float (&ct)[NT], const float (&tau)[NA][NT], float (&sl)[NA]) {
#pragma unroll
  for (int a = 0; a < NA; ++a) {
    float l = ct[0] * tau[a][0];
#pragma unroll
    for (int j = 1; j < NT; ++j) l = fmaf(ct[j], tau[a][j], l);
    sl[a] += l;
  }
}

// Terminal cost 1/2 tauN^T C_f tauN + c_f^T tauN with tauN = [x_T - xref_T; 0].
__device__ __forceinline__ float terminal_cost(const float* __restrict__ Cf, const float* __restrict__ cf,
                                               const float (&tn)[NX], bool ok) {
  if (Cf == nullptr || !ok) return 0.0f;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < NX; ++i) {
    float r = __ldg(Cf + i * NT) * tn[0];
#pragma unroll
    for (int j = 1; j < NX; ++j) r = fmaf(__ldg(Cf + i * NT + j), tn[j], r);
    q = fmaf(tn[i], r, q);
  }
  float l = 0.0f;
  if (cf != nullptr) {
    l = __ldg(cf) * tn[0];
#pragma unroll
    for (int i = 1; i < NX; ++i) l = fmaf(__ldg(cf + i), tn[i], l);
  }
  return 0.5f * q + l;
}

// Candidate control of the grid line search (controller.py:480-490):
// u = U_t + a k_t + a (K_t (x - X_t)), then max(., u_min), min(., u_max).
__device__ __forceinline__ void candidate_u(const float (&x)[NX], const float (&xb)[NX], const float (&ub)[NU],
                                            const float (&Kt)[NU][NX], const float (&kt)[NU], float al,
                                            bool bounds, const float (&lo)[NU], const float (&hi)[NU],
                                            float (&u)[NU]) {
  float dx[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) dx[i] = x[i] - xb[i];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    float kd = Kt[a][0] * dx[0];
#pragma unroll
    for (int i = 1; i < NX; ++i) kd = fmaf(Kt[a][i], dx[i], kd);
    float v = ub[a] + (al * kt[a] + al * kd);
    if (bounds) {
      v = (v != v) ? v : fmaxf(v, lo[a]);
      v = (v != v) ? v : fminf(v, hi[a]);
    }
    u[a] = v;
  }
}

template <int NAC, bool HAS_REF>
__global__ void __launch_bounds__(WARP) solve_kernel(const __grid_constant__ CUtensorMap tmC, const SolveParams p) {
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

  Ws ws;
  ws.S = S;
  ws.Xn = p.ws + b;
  ws.Un = p.ws + (int64_t)(T + 1) * NX * S + b;
  ws.K = ws.Un + (int64_t)T * NU * S;
  ws.k = ws.K + (int64_t)T * NU * NX * S;

  if (lane == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncwarp();
  CPipe pipe{cbuf, bar, 0u, &tmC, (int)b0};

  const bool bounds = p.has_bounds != 0;
  float lo[NU], hi[NU];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    lo[a] = bounds ? __ldg(p.u_min + a) : 0.0f;
    hi[a] = bounds ? __ldg(p.u_max + a) : 0.0f;
  }
  const float* cb = p.c + b * (int64_t)T * NT;
  const float* xrb = (HAS_REF && p.x_ref != nullptr) ? p.x_ref + b * (int64_t)(T + 1) * NX : nullptr;
  const float* urb = (HAS_REF && p.u_ref != nullptr) ? p.u_ref + b * (int64_t)T * NU : nullptr;
  auto xref = [&](int t, int i) { return (HAS_REF && xrb != nullptr) ? ldg_or0(xrb + t * NX + i, valid) : 0.0f; };
  auto uref = [&](int t, int a) { return (HAS_REF && urb != nullptr) ? ldg_or0(urb + t * NU + a, valid) : 0.0f; };
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;
  const float* cf = (p.c_f != nullptr && valid) ? p.c_f + b * NT : nullptr;

  float x0[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) x0[i] = ldg_or0(p.x0 + b * NX + i, valid);

  if (p.trace != nullptr && valid)
    for (int i = 0; i < p.max_iter; ++i) p.trace[b * p.max_iter + i] = (int8_t)-128;

  // ---- initial open-loop rollout with U_init (controller.py:305, 578-603) --
  {
    float x[NX];
#pragma unroll
    for (int i = 0; i < NX; ++i) x[i] = x0[i];
    for (int t = 0; t < T; ++t) {
      float u[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) u[a] = ldg_or0(p.U_init + (b * T + t) * NU + a, valid);
#pragma unroll
      for (int i = 0; i < NX; ++i) ws.x(t, i) = x[i];
#pragma unroll
      for (int a = 0; a < NU; ++a) ws.u(t, a) = u[a];
      float xn[NX];
      drone_step(x, u, dt, xn);
#pragma unroll
      for (int i = 0; i < NX; ++i) x[i] = xn[i];
    }
#pragma unroll
    for (int i = 0; i < NX; ++i) ws.x(T, i) = x[i];
  }

  uint32_t status = 0;
  bool pipe_ok = true;

  // ---- initial cost of the nominal trajectory (controller.py:308) ---------
  float best;
  {
    float sq[1] = {0.0f}, sl[1] = {0.0f};
    pipe_ok = pipe.run(T, false, [&](int t, const float* Crow) {
      float tau[1][NT], ct[NT];
#pragma unroll
      for (int i = 0; i < NX; ++i) tau[0][i] = ws.x(t, i) - xref(t, i);
#pragma unroll
      for (int a = 0; a < NU; ++a) tau[0][NX + a] = ws.u(t, a) - uref(t, a);
#pragma unroll
      for (int j = 0; j < NT; ++j) ct[j] = ldg_or0(cb + t * NT + j, valid);
      quad_accum<1>(Crow, tau, sq);
      lin_accum<1>(ct, tau, sl);
    });
    float tn[NX];
#pragma unroll
    for (int i = 0; i < NX; ++i) tn[i] = ws.x(T, i) - xref(T, i);
    best = (0.5f * sq[0] + sl[0]) + terminal_cost(Cf, cf, tn, valid);
  }

  bool active = valid && pipe_ok;
  int iters = 0;
  int stall_iter = p.max_iter;
  float stall_gap = 0.0f;

  for (int it = 0; it < p.max_iter; ++it) {
    if (p.forced != nullptr && active && p.forced[b * p.max_iter + it] == (int8_t)-128) active = false;
    if (!__any_sync(FULL, active)) break;

    // ---- backward Riccati pass (controller.py:315-318, 697-723) ------------
    float V[NX][NX], v[NX];
    {
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = ws.x(T, i) - xref(T, i);
#pragma unroll
      for (int i = 0; i < NX; ++i) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < NX; ++j) {
          const float cij = Cf ? __ldg(Cf + i * NT + j) : 0.0f;
          V[i][j] = cij;
          acc = fmaf(cij, tn[j], acc);
        }
        v[i] = acc + (cf ? __ldg(cf + i) : 0.0f);
      }
    }
    bool fallback = false;
    pipe_ok = pipe.run(T, true, [&](int t, const float* Crow) {
      float xb[NX], ub[NU], tau[NT];
#pragma unroll
      for (int i = 0; i < NX; ++i) {
        xb[i] = ws.x(t, i);
        tau[i] = xb[i] - xref(t, i);
      }
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        ub[a] = ws.u(t, a);
        tau[NX + a] = ub[a] - uref(t, a);
      }
      // quadraticize (cost.py:149-165): l_tau = C tau + c
      float lx[NX], lu[NU];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        float r = Crow[i * NT] * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) r = fmaf(Crow[i * NT + j], tau[j], r);
        r = r + ldg_or0(cb + t * NT + i, valid);
        if (i < NX) lx[i] = r; else lu[i - NX] = r;
      }
      const Jac J = drone_jac(xb, ub, dt);
      float K[NU][NX], k[NU];
      if (!riccati_step<false>(V, v, J, Crow, lx, lu, p.reg, 0u, K, k)) fallback = true;
#pragma unroll
      for (int a = 0; a < NU; ++a) {
#pragma unroll
        for (int j = 0; j < NX; ++j) ws.K_(t, a, j) = K[a][j];
        ws.k_(t, a) = k[a];
      }
    });
    if (!pipe_ok) { active = false; break; }
    if (fallback && active) status |= ELEM_CHOL_FALLBACK;

    // ---- grid line search (controller.py:360-388, 437-533) ----------------
    int jbest = 0;
    float cmin = 0.0f;
    bool have = false, nan_seen = false;
    float cand_cost[ILQR_MAX_ALPHAS_DEV];
    for (int a0 = 0; a0 < p.n_alpha; a0 += NAC) {
      float al[NAC];
#pragma unroll
      for (int a = 0; a < NAC; ++a) al[a] = (a0 + a < p.n_alpha) ? p.alphas[a0 + a] : 0.0f;
      float x[NAC][NX], sq[NAC], sl[NAC];
#pragma unroll
      for (int a = 0; a < NAC; ++a) {
        sq[a] = 0.0f;
        sl[a] = 0.0f;
#pragma unroll
        for (int i = 0; i < NX; ++i) x[a][i] = x0[i];
      }
      pipe_ok = pipe.run(T, false, [&](int t, const float* Crow) {
        float xb[NX], ub[NU], Kt[NU][NX], kt[NU], ct[NT];
#pragma unroll
        for (int i = 0; i < NX; ++i) xb[i] = ws.x(t, i);
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          ub[a] = ws.u(t, a);
          kt[a] = ws.k_(t, a);
#pragma unroll
          for (int j = 0; j < NX; ++j) Kt[a][j] = ws.K_(t, a, j);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) ct[j] = ldg_or0(cb + t * NT + j, valid);
        float xr[NX], ur[NU];
#pragma unroll
        for (int i = 0; i < NX; ++i) xr[i] = xref(t, i);
#pragma unroll
        for (int i = 0; i < NU; ++i) ur[i] = uref(t, i);
        float u[NAC][NU], tau[NAC][NT];
#pragma unroll
        for (int a = 0; a < NAC; ++a) {
          candidate_u(x[a], xb, ub, Kt, kt, al[a], bounds, lo, hi, u[a]);
#pragma unroll
          for (int i = 0; i < NX; ++i) tau[a][i] = x[a][i] - xr[i];
#pragma unroll
          for (int i = 0; i < NU; ++i) tau[a][NX + i] = u[a][i] - ur[i];
        }
        quad_accum<NAC>(Crow, tau, sq);
        lin_accum<NAC>(ct, tau, sl);
#pragma unroll
        for (int a = 0; a < NAC; ++a) {
          float xn[NX];
          drone_step(x[a], u[a], dt, xn);
#pragma unroll
          for (int i = 0; i < NX; ++i) x[a][i] = xn[i];
        }
      });
      if (!pipe_ok) break;
#pragma unroll
      for (int a = 0; a < NAC; ++a) {
        if (a0 + a >= p.n_alpha) continue;
        float tn[NX];
#pragma unroll
        for (int i = 0; i < NX; ++i) tn[i] = x[a][i] - xref(T, i);
        const float cost = (0.5f * sq[a] + sl[a]) + terminal_cost(Cf, cf, tn, valid);
        cand_cost[a0 + a] = cost;
        // torch.argmin semantics: the first NaN wins, else the first minimum.
        if (!nan_seen) {
          if (cost != cost) {
            nan_seen = true;
            jbest = a0 + a;
            cmin = cost;
          } else if (!have || cost < cmin) {
            have = true;
            jbest = a0 + a;
            cmin = cost;
          }
        }
      }
    }
    if (!pipe_ok) { active = false; break; }

    // ---- decision (controller.py:396-415) ---------------------------------
    bool accept = false;
    int jsel = jbest;
    if (active) {
      ++iters;
      if (p.forced != nullptr) {
        const int8_t d = p.forced[b * p.max_iter + it];
        if (d >= 0 && d < p.n_alpha) {
          accept = true;
          jsel = d;
        }
      } else {
        accept = cmin < best;
      }
      if (p.trace != nullptr) p.trace[b * p.max_iter + it] = (int8_t)(accept ? jsel : -(jbest + 1));
      if (!accept && stall_iter == p.max_iter) {
        stall_iter = it;
        stall_gap = fabsf(cmin - best);
      }
      if (accept) best = cand_cost[jsel];
      if (!accept && p.forced == nullptr) active = false;
    }
    // ---- re-run the accepted candidate, writing the new nominal ------------
    if (__any_sync(FULL, accept)) {
      const float al = p.alphas[jsel];
      float x[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) x[i] = x0[i];
      for (int t = 0; t < T; ++t) {
        float xb[NX], ub[NU], Kt[NU][NX], kt[NU], u[NU];
#pragma unroll
        for (int i = 0; i < NX; ++i) xb[i] = ws.x(t, i);
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          ub[a] = ws.u(t, a);
          kt[a] = ws.k_(t, a);
#pragma unroll
          for (int j = 0; j < NX; ++j) Kt[a][j] = ws.K_(t, a, j);
        }
        candidate_u(x, xb, ub, Kt, kt, al, bounds, lo, hi, u);
        if (accept) {
#pragma unroll
          for (int i = 0; i < NX; ++i) ws.x(t, i) = x[i];
#pragma unroll
          for (int a = 0; a < NU; ++a) ws.u(t, a) = u[a];
        }
        float xn[NX];
        drone_step(x, u, dt, xn);
#pragma unroll
        for (int i = 0; i < NX; ++i) x[i] = xn[i];
      }
      if (accept) {
#pragma unroll
        for (int i = 0; i < NX; ++i) ws.x(T, i) = x[i];
      }
    }
  }
  if (!pipe_ok) status |= ELEM_PIPE_TIMEOUT;

  // ---- outputs -------------------------------------------------------------
  if (!valid) return;
  bool finite = true;
  for (int t = 0; t <= T; ++t) {
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      const float xv = ws.x(t, i);
      finite &= isfinite(xv);
      p.X[(b * (T + 1) + t) * NX + i] = xv;
    }
  }
  for (int t = 0; t < T; ++t) {
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      const float uv = ws.u(t, a);
      finite &= isfinite(uv);
      p.U[(b * T + t) * NU + a] = uv;
      if (p.tight != nullptr) {
        // _compute_tight_mask (controller.py:997-1003): torch.isclose(U, bound,
        // rtol=1e-5, atol=1e-7) against u_min and u_max.
        bool tt = false;
        if (bounds) {
          const float e0 = fabsf(uv - lo[a]), e1 = fabsf(uv - hi[a]);
          tt = (uv == lo[a]) || (isfinite(e0) && e0 <= 1e-7f + fabsf(1e-5f * lo[a])) || (uv == hi[a]) ||
               (isfinite(e1) && e1 <= 1e-7f + fabsf(1e-5f * hi[a]));
        }
        p.tight[(b * T + t) * NU + a] = tt ? 1 : 0;
      }
    }
  }
  if (!finite) status |= ELEM_NONFINITE;
  if (p.iters) p.iters[b] = iters;
  if (p.status) p.status[b] = status;
  if (p.best_cost) p.best_cost[b] = best;
  if (p.stall_iter) p.stall_iter[b] = stall_iter;
  if (p.stall_gap) p.stall_gap[b] = stall_gap;
}

}  // namespace

size_t solve_smem_bytes() { return 2 * SLAB_BYTES + 2 * sizeof(uint64_t); }

cudaError_t launch_solve(const CUtensorMap& tmC, const SolveParams& p, cudaStream_t stream) {
  const size_t smem = solve_smem_bytes();
  const unsigned grid = (unsigned)((p.B + WARP - 1) / WARP);
  const bool ref = p.x_ref != nullptr || p.u_ref != nullptr;
  const bool four = (p.n_alpha % 4 == 0) && (p.n_alpha % 5 != 0);
#define ILQR_LAUNCH(NA, REF)                                                                       \
  do {                                                                                             \
    auto kfn = solve_kernel<NA, REF>;                                                              \
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                                \
    kfn<<<grid, WARP, smem, stream>>>(tmC, p);                                                     \
  } while (0)
  if (four) {
    if (ref) ILQR_LAUNCH(4, true); else ILQR_LAUNCH(4, false);
  } else {
    if (ref) ILQR_LAUNCH(5, true); else ILQR_LAUNCH(5, false);
  }
#undef ILQR_LAUNCH
  return cudaGetLastError();
}

}  // namespace ilqr
