// ilqr_solve.cu -- fused batched iLQR forward solve (all iterations, one launch).
//
// Mapping: one CTA = one warp = 6 batch elements, a team of 5 lanes per
// element (lanes 30, 31 are spare). The team splits each Riccati step by rows
// of V (ilqr_team.cuh) and evaluates the line-search step sizes one per lane.
// Per-element trajectories (nominal X, U) and gains (K, k) live in a
// caller-provided workspace, element-interleaved (field f of element b at
// ws[f * S + b]); the dense cost blocks C[b, t] of the warp's six elements are
// staged into shared memory by one TMA bulk tensor copy per step.
//
// Algorithm: DifferentiableMPCController.solve_step (controller.py:303-435)
// with per-element freezing: an element stops at its first non-improving
// iteration, which leaves X, U identical to the reference's global loop.
// The initial objective (controller.py:308) is accumulated during the first
// Riccati pass, which reads the same C_t blocks.
#include "ilqr_kernels.h"
#include "ilqr_team.cuh"

namespace ilqr {

namespace {

struct Ws {
  float* base;
  int64_t S;
  __device__ __forceinline__ float* x(int64_t b, int t, int i) const { return base + (int64_t)(t * NX + i) * S + b; }
};

__device__ __forceinline__ float ldg_or0(const float* p, bool ok) { return ok ? __ldg(p) : 0.0f; }

// Terminal cost 1/2 tauN^T C_f tauN + c_f^T tauN with tauN = [x_T - xref_T; 0].
__device__ __forceinline__ float terminal_cost(const float* __restrict__ Cf, const float* __restrict__ cf,
                                               const float (&tn)[NX]) {
  if (Cf == nullptr) return 0.0f;
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
// K_t rows are read from the workspace one at a time.
template <class KRow>
__device__ __forceinline__ void candidate_u(const float (&x)[NX], const float (&xb)[NX], const float (&ub)[NU],
                                            KRow&& krow, const float (&kt)[NU], float al,
                                            const float* __restrict__ lo, const float* __restrict__ hi,
                                            float (&u)[NU]) {
  float dx[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) dx[i] = x[i] - xb[i];
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    float Kr[NX];
    krow(a, Kr);
    float kd = Kr[0] * dx[0];
#pragma unroll
    for (int i = 1; i < NX; ++i) kd = fmaf(Kr[i], dx[i], kd);
    float v = ub[a] + (al * kt[a] + al * kd);
    if (lo != nullptr) {
      v = (v != v) ? v : fmaxf(v, __ldg(lo + a));
      v = (v != v) ? v : fminf(v, __ldg(hi + a));
    }
    u[a] = v;
  }
}

__device__ __forceinline__ float pick(const float (&v)[NT], int i) {
  float r = v[0];
#pragma unroll
  for (int j = 1; j < NT; ++j) r = (i == j) ? v[j] : r;
  return r;
}

template <int NAC, bool HAS_REF>
__global__ void __launch_bounds__(32, 19) solve_kernel(const __grid_constant__ CUtensorMap tmC,
                                                       const SolveParams p) {
  static_assert(NAC == TEAM, "one step size per team lane");
  extern __shared__ __align__(128) unsigned char smem[];
  float* slab = reinterpret_cast<float*>(smem);
  float* xch = slab + SLAB_E * CBLK;
  uint64_t* bar = reinterpret_cast<uint64_t*>(xch + SLAB_E * XS);
  const int lane = threadIdx.x;
  const int e = lane / TEAM;
  const int m = lane - e * TEAM;
  const int base = e * TEAM;
  const int64_t b0 = (int64_t)blockIdx.x * EPW;
  const int64_t b = b0 + e;
  const bool valid = (e < EPW) && (b < p.B);
  const int64_t bw = valid ? b : b0;  // workspace slot read by this lane (never written when !valid)
  const int T = p.T;
  const float dt = p.dt;
  const Ws ws{p.ws, p.S};
  float* Kw = p.ws + (int64_t)((T + 1) * NX + T * NU) * p.S;
  float* kw = Kw + (int64_t)T * NU * NX * p.S;
  auto Xn = [&](int t, int i) -> float& { return *ws.x(bw, t, i); };
  auto Un = [&](int t, int a) -> float& { return p.ws[(int64_t)((T + 1) * NX + t * NU + a) * p.S + bw]; };
  auto Kat = [&](int t, int a, int j) -> float& { return Kw[(int64_t)(t * NU * NX + a * NX + j) * p.S + bw]; };
  auto kat = [&](int t, int a) -> float& { return kw[(int64_t)(t * NU + a) * p.S + bw]; };

  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  TeamPipe pipe{slab, bar, 0u, &tmC, (int)b0, true};
  float* xc = xch + e * XS;
  const float* Ce = slab + e * CBLK;
  const int ra = row_a(m), rb = row_b(m);

  const bool bounds = p.has_bounds != 0;
  const float* lo = bounds ? p.u_min : nullptr;
  const float* hi = bounds ? p.u_max : nullptr;
  const float* cb = p.c + b * (int64_t)T * NT;
  const float* xrb = (HAS_REF && p.x_ref != nullptr) ? p.x_ref + b * (int64_t)(T + 1) * NX : nullptr;
  const float* urb = (HAS_REF && p.u_ref != nullptr) ? p.u_ref + b * (int64_t)T * NU : nullptr;
  auto xref = [&](int t, int i) { return (HAS_REF && xrb != nullptr) ? ldg_or0(xrb + t * NX + i, valid) : 0.0f; };
  auto uref = [&](int t, int a) { return (HAS_REF && urb != nullptr) ? ldg_or0(urb + t * NU + a, valid) : 0.0f; };
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;
  const float* cf = (p.c_f != nullptr && valid) ? p.c_f + b * NT : nullptr;

  auto load_x0 = [&](float (&x)[NX]) {
#pragma unroll
    for (int i = 0; i < NX; ++i) x[i] = ldg_or0(p.x0 + b * NX + i, valid);
  };
  const bool writer = valid && m == 0;
  if (p.trace != nullptr && writer)
    for (int i = 0; i < p.max_iter; ++i) p.trace[b * p.max_iter + i] = (int8_t)-128;

  // ---- initial open-loop rollout with U_init (controller.py:305, 578-603) --
  {
    float x[NX];
    load_x0(x);
    for (int t = 0; t < T; ++t) {
      float u[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) u[a] = ldg_or0(p.U_init + (b * T + t) * NU + a, valid);
      if (writer) {
#pragma unroll
        for (int i = 0; i < NX; ++i) Xn(t, i) = x[i];
#pragma unroll
        for (int a = 0; a < NU; ++a) Un(t, a) = u[a];
      }
      float xn[NX];
      drone_step(x, u, dt, xn);
#pragma unroll
      for (int i = 0; i < NX; ++i) x[i] = xn[i];
    }
    if (writer) {
#pragma unroll
      for (int i = 0; i < NX; ++i) Xn(T, i) = x[i];
    }
  }
  __syncwarp();

  uint32_t status = 0;
  bool active = valid;
  int iters = 0;
  int stall_iter = p.max_iter;
  float stall_gap = 0.0f;
  float best = 0.0f;

  // The first pass always runs: it also yields the initial objective (with
  // max_iter == 0 only that).
  const int n_loop = p.max_iter > 0 ? p.max_iter : 1;
  for (int it = 0; it < n_loop; ++it) {
    const bool cost_only = it >= p.max_iter;
    if (!cost_only && p.forced != nullptr && active && p.forced[b * p.max_iter + it] == (int8_t)-128)
      active = false;
    if (!__any_sync(FULL, active) && it > 0) break;

    // ---- backward Riccati pass (controller.py:315-318, 697-723) ------------
    float Va[NX], Vb[NX], va_, vb_;
    {
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = Xn(T, i) - xref(T, i);
      float acca = 0.0f, accb = 0.0f;
#pragma unroll
      for (int j = 0; j < NX; ++j) {
        Va[j] = Cf ? __ldg(Cf + ra * NT + j) : 0.0f;
        Vb[j] = Cf ? __ldg(Cf + rb * NT + j) : 0.0f;
        acca = fmaf(Va[j], tn[j], acca);
        accb = fmaf(Vb[j], tn[j], accb);
      }
      va_ = acca + (cf ? __ldg(cf + ra) : 0.0f);
      vb_ = accb + (cf ? __ldg(cf + rb) : 0.0f);
    }
    bool fallback = false;
    float cost_q = 0.0f, cost_l = 0.0f;  // initial objective, first pass only
    const bool first = (it == 0);
    bool ok = pipe.run(T, true, [&](int t, auto&& next) {
      float xb[NX], ub[NU], tau[NT], ct[NT];
#pragma unroll
      for (int i = 0; i < NX; ++i) {
        xb[i] = Xn(t, i);
        tau[i] = xb[i] - xref(t, i);
      }
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        ub[a] = Un(t, a);
        tau[NX + a] = ub[a] - uref(t, a);
      }
      // quadraticize my rows (cost.py:149-165): l_tau = C tau + c
      auto rowdot = [&](int r) {
        const float* Cr = Ce + r * NT;
        float s = Cr[0] * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) s = fmaf(Cr[j], tau[j], s);
        return s;
      };
      const float ca_ = ldg_or0(cb + t * NT + ra, valid), cb_ = ldg_or0(cb + t * NT + rb, valid);
      const float sa = rowdot(ra), sb = rowdot(rb);
      const float lxa = sa + ca_, lxb = sb + cb_;
      const int ru = NX + (m < NU ? m : 0);
      const float su = rowdot(ru), cu = ldg_or0(cb + t * NT + ru, valid);
      if (m < NU) xc[X_LU + m] = su + cu;
      if (first) {
        const float ta = pick(tau, ra), tb = pick(tau, rb), tu = pick(tau, ru);
        cost_q += fmaf(ta, sa, tb * sb) + (m < NU ? tu * su : 0.0f);
        cost_l += fmaf(ca_, ta, cb_ * tb) + (m < NU ? cu * tu : 0.0f);
      }
      __syncwarp();
      const Jac J = drone_jac(xb, ub, dt);
      float Ka[NU], Kb[NU], k[NU];
      if (!team_riccati<false>(Va, Vb, va_, vb_, J, DenseC{Ce}, lxa, lxb, p.reg, 0u, m, xc, next, Ka, Kb, k))
        fallback = true;
      if (valid) {
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          Kat(t, a, ra) = Ka[a];
          Kat(t, a, rb) = Kb[a];
        }
        if (m == 0) {
#pragma unroll
          for (int a = 0; a < NU; ++a) kat(t, a) = k[a];
        }
      }
    });
    if (!ok) {
      status |= ELEM_PIPE_TIMEOUT;
      active = false;
      break;
    }
    if (team_sum(fallback ? 1.0f : 0.0f, base) > 0.0f && active) status |= ELEM_CHOL_FALLBACK;
    if (first) {
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = Xn(T, i) - xref(T, i);
      best = (0.5f * team_sum(cost_q, base) + team_sum(cost_l, base)) + terminal_cost(Cf, cf, tn);
    }
    __syncwarp();
    if (cost_only) break;

    // ---- grid line search (controller.py:360-388, 437-533): lane m = step m --
    int jbest = 0;
    float cmin = 0.0f;
    bool have = false, nan_seen = false;
    float cand[ILQR_MAX_ALPHAS_DEV];
    for (int a0 = 0; a0 < p.n_alpha; a0 += NAC) {
      const float al = (a0 + m < p.n_alpha) ? p.alphas[a0 + m] : 0.0f;
      float x[NX], sq = 0.0f, sl = 0.0f;
      load_x0(x);
      ok = pipe.run(T, false, [&](int t, auto&& next) {
        float xb[NX], ub[NU], kt[NU], u[NU];
#pragma unroll
        for (int i = 0; i < NX; ++i) xb[i] = Xn(t, i);
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          ub[a] = Un(t, a);
          kt[a] = kat(t, a);
        }
        candidate_u(x, xb, ub,
                    [&](int a, float (&Kr)[NX]) {
#pragma unroll
                      for (int j = 0; j < NX; ++j) Kr[j] = Kat(t, a, j);
                    },
                    kt, al, lo, hi, u);
        float tau[NT];
#pragma unroll
        for (int i = 0; i < NX; ++i) tau[i] = x[i] - xref(t, i);
#pragma unroll
        for (int a = 0; a < NU; ++a) tau[NX + a] = u[a] - uref(t, a);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          const float2* r2 = reinterpret_cast<const float2*>(Ce + i * NT);
          float r = 0.0f;
#pragma unroll
          for (int j = 0; j < NT / 2; ++j) {
            const float2 c2 = r2[j];
            r = (j == 0) ? c2.x * tau[0] : fmaf(c2.x, tau[2 * j], r);
            r = fmaf(c2.y, tau[2 * j + 1], r);
          }
          q = fmaf(tau[i], r, q);
        }
        next();
        float l = ldg_or0(cb + t * NT, valid) * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) l = fmaf(ldg_or0(cb + t * NT + j, valid), tau[j], l);
        sq += q;
        sl += l;
        float xn[NX];
        drone_step(x, u, dt, xn);
#pragma unroll
        for (int i = 0; i < NX; ++i) x[i] = xn[i];
      });
      if (!ok) break;
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = x[i] - xref(T, i);
      const float mine = (0.5f * sq + sl) + terminal_cost(Cf, cf, tn);
      // gather the team's costs; torch.argmin semantics (first NaN, else first minimum)
#pragma unroll
      for (int j = 0; j < NAC; ++j) {
        const float cj = __shfl_sync(FULL, mine, (base + j) & 31);
        if (a0 + j >= p.n_alpha) continue;
        cand[a0 + j] = cj;
        if (!nan_seen) {
          if (cj != cj) {
            nan_seen = true;
            jbest = a0 + j;
            cmin = cj;
          } else if (!have || cj < cmin) {
            have = true;
            jbest = a0 + j;
            cmin = cj;
          }
        }
      }
    }
    if (!ok) {
      status |= ELEM_PIPE_TIMEOUT;
      active = false;
      break;
    }

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
      if (p.trace != nullptr && m == 0) p.trace[b * p.max_iter + it] = (int8_t)(accept ? jsel : -(jbest + 1));
      if (!accept && stall_iter == p.max_iter) {
        stall_iter = it;
        stall_gap = fabsf(cmin - best);
      }
      if (accept) best = cand[jsel];
      if (!accept && p.forced == nullptr) active = false;
    }
    // ---- lane 0 re-runs the accepted candidate, writing the new nominal -----
    if (__any_sync(FULL, accept)) {
      if (accept && m == 0) {
        const float al = p.alphas[jsel];
        float x[NX];
        load_x0(x);
        for (int t = 0; t < T; ++t) {
          float xb[NX], ub[NU], kt[NU], u[NU];
#pragma unroll
          for (int i = 0; i < NX; ++i) xb[i] = Xn(t, i);
#pragma unroll
          for (int a = 0; a < NU; ++a) {
            ub[a] = Un(t, a);
            kt[a] = kat(t, a);
          }
          candidate_u(x, xb, ub,
                      [&](int a, float (&Kr)[NX]) {
#pragma unroll
                        for (int j = 0; j < NX; ++j) Kr[j] = Kat(t, a, j);
                      },
                      kt, al, lo, hi, u);
#pragma unroll
          for (int i = 0; i < NX; ++i) Xn(t, i) = x[i];
#pragma unroll
          for (int a = 0; a < NU; ++a) Un(t, a) = u[a];
          float xn[NX];
          drone_step(x, u, dt, xn);
#pragma unroll
          for (int i = 0; i < NX; ++i) x[i] = xn[i];
        }
#pragma unroll
        for (int i = 0; i < NX; ++i) Xn(T, i) = x[i];
      }
      __syncwarp();
    }
  }

  // ---- outputs (lanes of a team split the writes) -----------------------------
  bool finite = true;
  if (valid) {
    for (int f = m; f < (T + 1) * NX; f += TEAM) {
      const float xv = *ws.x(bw, 0, f);
      finite &= isfinite(xv);
      p.X[b * (T + 1) * NX + f] = xv;
    }
    for (int f = m; f < T * NU; f += TEAM) {
      const int t = f / NU, a = f - t * NU;
      const float uv = Un(t, a);
      finite &= isfinite(uv);
      p.U[b * T * NU + f] = uv;
      if (p.tight != nullptr) {
        // _compute_tight_mask (controller.py:997-1003): torch.isclose(U, bound,
        // rtol=1e-5, atol=1e-7) against u_min and u_max.
        bool tt = false;
        if (bounds) {
          const float l_ = __ldg(lo + a), h_ = __ldg(hi + a);
          const float e0 = fabsf(uv - l_), e1 = fabsf(uv - h_);
          tt = (uv == l_) || (isfinite(e0) && e0 <= 1e-7f + fabsf(1e-5f * l_)) || (uv == h_) ||
               (isfinite(e1) && e1 <= 1e-7f + fabsf(1e-5f * h_));
        }
        p.tight[b * T * NU + f] = tt ? 1 : 0;
      }
    }
  }
  const bool all_finite = team_sum(finite ? 0.0f : 1.0f, base) == 0.0f;
  if (!all_finite) status |= ELEM_NONFINITE;
  if (writer) {
    if (p.iters) p.iters[b] = iters;
    if (p.status) p.status[b] = status;
    if (p.best_cost) p.best_cost[b] = best;
    if (p.stall_iter) p.stall_iter[b] = stall_iter;
    if (p.stall_gap) p.stall_gap[b] = stall_gap;
  }
}

}  // namespace

size_t solve_smem_bytes() { return (size_t)SLAB_E * CBLK * 4 + (size_t)SLAB_E * XS * 4 + sizeof(uint64_t); }

cudaError_t launch_solve(const CUtensorMap& tmC, const SolveParams& p, cudaStream_t stream) {
  const size_t smem = solve_smem_bytes();
  const unsigned grid = (unsigned)((p.B + EPW - 1) / EPW);
  const bool ref = p.x_ref != nullptr || p.u_ref != nullptr;
  if (ref) {
    solve_kernel<TEAM, true><<<grid, WARP, smem, stream>>>(tmC, p);
  } else {
    solve_kernel<TEAM, false><<<grid, WARP, smem, stream>>>(tmC, p);
  }
  return cudaGetLastError();
}

}  // namespace ilqr
