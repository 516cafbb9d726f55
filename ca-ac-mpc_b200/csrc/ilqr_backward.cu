// ilqr_backward.cu -- fused implicit-differentiation backward pass.
//
// One CTA = one warp = 6 batch elements, a 5-lane team per element (as the
// solve kernel). Two passes over the horizon:
//   1. reverse: masked adjoint Riccati (controller.py:1035-1110) split by rows
//      of V across the team (ilqr_team.cuh), A_t, B_t recomputed from
//      (X_t, U_t), l_xx / l_xu / l_uu read from the TMA-staged C_t slab; the
//      gains go to an element-interleaved workspace (one float4 per column of
//      K_t and one for k_t).
//   2. forward: dU = K dX + k, dX+ = A dX + B dU (controller.py:1121-1129),
//      computed by every lane of the team, and the gradients of
//      ILQRSolve.backward (controller.py:84-125) with the rows of grad_C[b, t]
//      split across the team, written into the shared-memory slab and stored
//      with one TMA bulk tensor store per step for the warp's six elements.
#include "ilqr_kernels.h"
#include "ilqr_pair.cuh"
#include "ilqr_team.cuh"

namespace ilqr {

namespace {

__device__ __forceinline__ float pick14(const float (&v)[NT], int i) {
  float r = v[0];
#pragma unroll
  for (int j = 1; j < NT; ++j) r = (i == j) ? v[j] : r;
  return r;
}

template <int MINB>
__global__ void __launch_bounds__(32, MINB) backward_kernel(const __grid_constant__ CUtensorMap tmC,
                                                          const __grid_constant__ CUtensorMap tmG,
                                                          const BackwardParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* slab = reinterpret_cast<float*>(smem);
  float* xch = slab + EPW * CBLK;
  uint64_t* bar = reinterpret_cast<uint64_t*>(xch + EPW * XS);
  const int lane = threadIdx.x;
  // Lanes 30, 31 mirror lanes 25, 26 (element 5, members 0 and 1): same loads
  // and arithmetic, bit-identical shared-memory writes, no global writes.
  const bool dup = lane >= EPW * TEAM;
  const int e = dup ? EPW - 1 : lane / TEAM;
  const int m = lane - (dup ? EPW * TEAM : e * TEAM);
  const int64_t b0 = (int64_t)blockIdx.x * EPW;
  const int64_t b = b0 + e;
  const bool valid = b < p.B;
  const bool own = valid && !dup;
  const int64_t bw = valid ? b : b0;
  const int T = p.T;
  const float dt = p.dt;
  // workspace: K_t columns [T][10][S][4] (the 4 gains of state j), k_t [T][S][4]
  auto kcol = [&](int t, int j) {
    return reinterpret_cast<float4*>(p.ws + ((size_t)(t * NX + j) * (size_t)p.S + (size_t)bw) * 4);
  };
  auto kff = [&](int t) {
    return reinterpret_cast<float4*>(p.ws + ((size_t)T * NX * (size_t)p.S + (size_t)t * p.S + (size_t)bw) * 4);
  };
  auto f4 = [](const float (&v)[NU]) { return make_float4(v[0], v[1], v[2], v[3]); };
  auto ld = [&](const float* q, int64_t i) { return valid ? __ldg(q + i) : 0.0f; };

  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  TeamPipe pipe{slab, bar, 0u, &tmC, (int)b0, true};
  float* xc = xch + e * XS;
  float* Ce = slab + e * CBLK;
  const int ra = row_a(m), rb = row_b(m);

  const float* Xb = p.X + b * (int64_t)(T + 1) * NX;
  const float* Ub = p.U + b * (int64_t)T * NU;
  const float* gXb = p.gX + b * (int64_t)(T + 1) * NX;
  const float* gUb = p.gU + b * (int64_t)T * NU;
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;

  // ---- 1. masked adjoint Riccati, V_T = C_f[:nx,:nx], v_T = -dL/dX_T --------
  float Va[NX], Vb[NX];
  float va_ = -ld(gXb, T * NX + ra), vb_ = -ld(gXb, T * NX + rb);
#pragma unroll
  for (int j = 0; j < NX; ++j) {
    Va[j] = Cf ? __ldg(Cf + ra * NT + j) : 0.0f;
    Vb[j] = Cf ? __ldg(Cf + rb * NT + j) : 0.0f;
  }
  // Costs from policy parameters: the slab holds zeros off the diagonal and
  // each step's diagonal is built from the parameters instead of copied.
  const bool sigm = p.sig.p != nullptr;
  const float* sgrow = sigm ? p.sig.p + bw * (int64_t)(2 * NT) * T : nullptr;
  if (sigm) {
    for (int f = lane; f < EPW * CBLK; f += WARP) slab[f] = 0.0f;
    __syncwarp();
  }
  auto sig_fill = [&](int t) {
#pragma unroll
    for (int s3 = 0; s3 < 3; ++s3) {
      const int i = m + TEAM * s3;
      if (i < NT) Ce[i * (NT + 1)] = sig_diag(p.sig, sgrow, T, t, i);
    }
  };
  bool ok = pipe.run(T, true, !sigm, sig_fill, [&](int t, auto&& next) {
    float xb[NX], ub[NU];
#pragma unroll
    for (int i = 0; i < NX; ++i) xb[i] = ld(Xb, t * NX + i);
#pragma unroll
    for (int a = 0; a < NU; ++a) ub[a] = ld(Ub, t * NU + a);
    const float lxa = -ld(gXb, t * NX + ra), lxb = -ld(gXb, t * NX + rb);
    if (m < NU) xc[X_LU + m] = -ld(gUb, t * NU + m);
    uint32_t tight = 0;
    if (p.tight != nullptr && valid) {
#pragma unroll
      for (int a = 0; a < NU; ++a) tight |= (p.tight[(b * T + t) * NU + a] != 0 ? 1u : 0u) << a;
    }
    __syncwarp();
    const Jac J = drone_jac(xb, ub, dt);
    float Ka[NU], Kb[NU], k[NU];
    team_riccati<true, (MINB < TIER_LO)>(Va, Vb, va_, vb_, J, DenseC{Ce}, lxa, lxb, p.reg, tight, m, valid, xc, next,
                                         Ka, Kb, k);
    if (own) {
      *kcol(t, ra) = f4(Ka);
      *kcol(t, rb) = f4(Kb);
      if (m == 0) *kff(t) = f4(k);
    }
  });
  if (!ok) return;  // a bounded wait gave up; outputs are left untouched
  if (own && p.g_x0 != nullptr) {
    p.g_x0[b * NX + ra] = -va_;
    p.g_x0[b * NX + rb] = -vb_;
  }
  __syncwarp();

  // ---- 2. tangent sweep and gradient assembly -------------------------------
  float dx[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) dx[i] = 0.0f;
  const int nrows = (m < NT - 2 * TEAM) ? 3 : 2;  // rows m, m+5, m+10 of grad_C
  for (int t = 0; t < T; ++t) {
    float z[NT], du[NU];
#pragma unroll
    for (int i = 0; i < NX; ++i) z[i] = ld(Xb, t * NX + i);
#pragma unroll
    for (int a = 0; a < NU; ++a) z[NX + a] = ld(Ub, t * NU + a);
    {
      // dU = K dX + k, each row accumulated over j in index order
      float4 c = *kcol(t, 0);
      float acc[NU] = {c.x * dx[0], c.y * dx[0], c.z * dx[0], c.w * dx[0]};
#pragma unroll
      for (int j = 1; j < NX; ++j) {
        c = *kcol(t, j);
        acc[0] = fmaf(c.x, dx[j], acc[0]);
        acc[1] = fmaf(c.y, dx[j], acc[1]);
        acc[2] = fmaf(c.z, dx[j], acc[2]);
        acc[3] = fmaf(c.w, dx[j], acc[3]);
      }
      const float4 kk = *kff(t);
      du[0] = acc[0] + kk.x;
      du[1] = acc[1] + kk.y;
      du[2] = acc[2] + kk.z;
      du[3] = acc[3] + kk.w;
    }
    float dtau[NT];
#pragma unroll
    for (int i = 0; i < NX; ++i) dtau[i] = dx[i];
#pragma unroll
    for (int a = 0; a < NU; ++a) dtau[NX + a] = du[a];
    if (p.write_gC) {
      if (t > 0) {
        if (lane == 0) bulk_wait_read<0>();  // previous step's store has read the slab
        __syncwarp();
      }
      // grad_C = -1/2 (dtau (x) z + z (x) dtau), z = [X_t; U_t] (controller.py:87-96)
      for (int s = 0; s < nrows; ++s) {
        const int i = m + TEAM * s;
        const float di = pick14(dtau, i), zi = pick14(z, i);
        float2* row = reinterpret_cast<float2*>(Ce + i * NT);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          const float g0 = -0.5f * (di * z[j] + zi * dtau[j]);
          const float g1 = -0.5f * (di * z[j + 1] + zi * dtau[j + 1]);
          row[j / 2] = make_float2(g0, g1);
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tmG, slab, 0, t, (int)b0);
        bulk_commit();
      }
    }
    if (own && sigm && p.g_sig != nullptr) {
      // gradient of the parameters through _build_cost_tensors: dL/dx_q =
      // grad_C[t,i,i] range_q, dL/dx_p = grad_c[t,i] range_p, and for the
      // thrust entry c = -(x_p range_pt + eps): dL/dx_p = -grad_c range_pt
      float* gq = p.g_sig + b * (int64_t)(2 * NT) * T;
      for (int s = 0; s < nrows; ++s) {
        const int i = m + TEAM * s;
        const float di = pick14(dtau, i), zi = pick14(z, i);
        const float gii = -0.5f * (di * zi + zi * di);
        const int off = sig_off(T, t, i);
        gq[off] = gii * p.sig.range_q;
        const float gc = -di;
        gq[14 * T + off] = i == NX ? (-gc) * p.sig.range_pt : gc * p.sig.range_p;
      }
    }
    if (own) {
      for (int s = 0; s < nrows; ++s) {
        const int i = m + TEAM * s;
        const float di = pick14(dtau, i);
        if (p.g_c != nullptr) p.g_c[b * p.gc_bstride + t * p.gc_tstride + i] = -di;
        if (i < NX && p.g_xref != nullptr) p.g_xref[(b * (T + 1) + t) * NX + i] = di;
        if (i >= NX && p.g_uref != nullptr) p.g_uref[(b * T + t) * NU + (i - NX)] = di;
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
  if (!own) return;
  if (p.g_xref != nullptr && m == 0) {
#pragma unroll
    for (int i = 0; i < NX; ++i) p.g_xref[(b * (T + 1) + T) * NX + i] = 0.0f;
  }
  if (p.g_Cf != nullptr || p.g_cf != nullptr) {
    float ev[NX];
#pragma unroll
    for (int i = 0; i < NX; ++i)
      ev[i] = ld(Xb, T * NX + i) - (p.x_ref != nullptr ? __ldg(p.x_ref + (b * (T + 1) + T) * NX + i) : 0.0f);
    if (p.g_Cf != nullptr) {
      for (int f = m; f < CBLK; f += TEAM) {
        const int i = f / NT, j = f - i * NT;
        float g = 0.0f;
        if (i < NX && j < NX) {
          float di = 0.0f, dj = 0.0f, ei = 0.0f, ej = 0.0f;
#pragma unroll
          for (int q = 0; q < NX; ++q) {
            if (q == i) { di = dx[q]; ei = ev[q]; }
            if (q == j) { dj = dx[q]; ej = ev[q]; }
          }
          g = -0.5f * (di * ej + ei * dj);
        }
        p.g_Cf[b * CBLK + f] = g;
      }
    }
    if (p.g_cf != nullptr && m == 0) {
#pragma unroll
      for (int i = 0; i < NT; ++i) p.g_cf[b * NT + i] = i < NX ? -dx[i] : 0.0f;
    }
  }
}


__device__ __forceinline__ void load_rec4(const float* r, float (&x)[NX], float (&u)[NU]) {
  const float4* q = reinterpret_cast<const float4*>(r);
  const float4 a = q[0], c = q[1], d = q[2], e = q[3];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  x[8] = d.x; x[9] = d.y; u[0] = d.z; u[1] = d.w;
  u[2] = e.x; u[3] = e.y;
}

// Bulk copy of `bytes` (a multiple of 16) from shared to global memory,
// completion tracked by the issuing thread's bulk groups.
__device__ __forceinline__ void bulk_store(float* dst, const float* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}

// The pair layout of the same backward (ilqr_pair.cuh): one element per
// half-warp; lane i < 10 owns row i of V in the masked Riccati pass, lane
// i < 14 row i of grad_C[b, t] in the sweep. grad_C rows go to a
// double-buffered staging block in shared memory and each block is stored
// with one bulk copy (784 contiguous bytes). Same formulas and order as the
// team kernel, so the same bits.
template <int MINB>
__global__ void __launch_bounds__(32, MINB) backward_pair_kernel(const BackwardParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x;
  const int h = lane >> 4, i = lane & (HALF - 1);
  const int64_t b0 = (int64_t)blockIdx.x * EPWP;
  const int64_t b = b0 + h;
  const bool valid = b < p.B;
  const int64_t bw = valid ? b : b0;
  const int T = p.T;
  const float dt = p.dt;
  float* sh = reinterpret_cast<float*>(smem) + h * pair_area(T, PREC_F + PJT_F + PKS_F + PLX_F);
  float* REC = sh + PBASE;         // [T][16] X_t, U_t
  float* JT = REC + PREC_F * T;    // [T][32] Jacobian tables
  float* KS = JT + PJT_F * T;      // [T][44] K columns, then k
  float* LX = KS + PKS_F * T;      // [T][16] -dL/dX_t (10), -dL/dU_t (4), the tight bits
  int own;
  const uint64_t coffs = pair_coef_offsets(i < NT ? i : NT - 1, own);
  auto f4 = [](const float (&v)[NU]) { return make_float4(v[0], v[1], v[2], v[3]); };
  auto ld = [&](const float* q, int64_t k) { return valid ? __ldg(q + k) : 0.0f; };
  const float* Xb = p.X + b * (int64_t)(T + 1) * NX;
  const float* Ub = p.U + b * (int64_t)T * NU;
  const float* gXb = p.gX + b * (int64_t)(T + 1) * NX;
  const float* gUb = p.gU + b * (int64_t)T * NU;
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;
  const int ri = i < NX ? i : 0;

  // ---- 1. masked adjoint Riccati, V_T = C_f[:nx,:nx], v_T = -dL/dX_T --------
  float Vr[NX];
  float vr = -ld(gXb, T * NX + ri);
#pragma unroll
  for (int j = 0; j < NX; ++j) Vr[j] = Cf ? __ldg(Cf + ri * NT + j) : 0.0f;
  const bool sigm = p.sig.p != nullptr;
  const float* sgrow = sigm ? p.sig.p + bw * (int64_t)(2 * NT) * T : nullptr;
  PairCPipe cpipe{sigm ? nullptr : p.C + bw * p.C_bstride * CBLK, p.C_tstride, sh + PC0, i};
  if (sigm) {
    for (int f = i; f < CBLK; f += HALF) sh[PC0 + f] = 0.0f;
  } else {
    cpipe.issue(T - 1);
  }
  // prologue: every step's (X_t, U_t) and Jacobian table, a step per lane
  for (int t = i; t < T; t += HALF) {
    float xb[NX], ub[NU];
#pragma unroll
    for (int k = 0; k < NX; ++k) xb[k] = ld(Xb, t * NX + k);
#pragma unroll
    for (int a = 0; a < NU; ++a) ub[a] = ld(Ub, t * NU + a);
    float4* d4 = reinterpret_cast<float4*>(REC + PREC_F * t);
    d4[0] = make_float4(xb[0], xb[1], xb[2], xb[3]);
    d4[1] = make_float4(xb[4], xb[5], xb[6], xb[7]);
    d4[2] = make_float4(xb[8], xb[9], ub[0], ub[1]);
    d4[3] = make_float4(ub[2], ub[3], 0.0f, 0.0f);
    jtab_write(JT + PJT_F * t, drone_jac(xb, ub, dt));
    float* lxt = LX + PLX_F * t;
#pragma unroll
    for (int k = 0; k < NX; ++k) lxt[k] = -ld(gXb, t * NX + k);
#pragma unroll
    for (int a = 0; a < NU; ++a) lxt[NX + a] = -ld(gUb, t * NU + a);
    uint32_t tb = 0;
    if (p.tight != nullptr && valid) {
#pragma unroll
      for (int a = 0; a < NU; ++a) tb |= (p.tight[(b * T + t) * NU + a] != 0 ? 1u : 0u) << a;
    }
    lxt[NT] = __uint_as_float(tb);
  }
  __syncwarp();
  for (int t = T - 1; t >= 0; --t) {
    const float* lxt = LX + PLX_F * t;
    const float lx = i < NT ? lxt[i] : 0.0f;
    const uint32_t tight = __float_as_uint(lxt[NT]);
    if (sigm) {
      if (i < NT) sh[PC0 + i * (NT + 1)] = sig_diag(p.sig, sgrow, T, t, i);
    } else if (t > 0) {
      cpipe.issue(t - 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const float* jt = JT + PJT_F * t;
    const Jac J = jtab_read(jt);
    float cf_[7], c7;
    pair_coef_load(jt, coffs, cf_, c7);
    __syncwarp();
    float Kr[NU];
    pair_riccati<true>(Vr, vr, J, cf_, c7, own, sigm ? sh + PC0 : cpipe.block(t), [&] { return lx; }, p.reg, tight,
                       i, valid, sh,
                       Kr);
    if (i <= NX) *reinterpret_cast<float4*>(KS + PKS_F * t + 4 * i) = f4(Kr);
  }
  if (valid && p.g_x0 != nullptr && i < NX) p.g_x0[b * NX + i] = -vr;
  __syncwarp();

  // ---- 2. tangent sweep and gradient assembly -------------------------------
  // grad_C[b, t] staging: two blocks of 196 floats at the start of the area
  // (the C_t buffers, free now); block t goes out with one bulk copy by lane 0
  // of the half, and block t - 2's copy must have read its buffer first.
  float dx[NX];
#pragma unroll
  for (int k = 0; k < NX; ++k) dx[k] = 0.0f;
  const bool wgc = p.write_gC && valid;
  float* gCb = wgc ? p.g_C + b * p.C_bstride * CBLK : nullptr;
  for (int t = 0; t < T; ++t) {
    float z[NT], du[NU];
    {
      float xz[NX], uz[NU];
      load_rec4(REC + PREC_F * t, xz, uz);
#pragma unroll
      for (int k = 0; k < NX; ++k) z[k] = xz[k];
#pragma unroll
      for (int a = 0; a < NU; ++a) z[NX + a] = uz[a];
    }
    const float4* ks = reinterpret_cast<const float4*>(KS + PKS_F * t);
    {
      float4 c = ks[0];
      float acc[NU] = {c.x * dx[0], c.y * dx[0], c.z * dx[0], c.w * dx[0]};
#pragma unroll
      for (int j = 1; j < NX; ++j) {
        c = ks[j];
        acc[0] = fmaf(c.x, dx[j], acc[0]);
        acc[1] = fmaf(c.y, dx[j], acc[1]);
        acc[2] = fmaf(c.z, dx[j], acc[2]);
        acc[3] = fmaf(c.w, dx[j], acc[3]);
      }
      const float4 kk = ks[NX];
      du[0] = acc[0] + kk.x;
      du[1] = acc[1] + kk.y;
      du[2] = acc[2] + kk.z;
      du[3] = acc[3] + kk.w;
    }
    float dtau[NT];
#pragma unroll
    for (int k = 0; k < NX; ++k) dtau[k] = dx[k];
#pragma unroll
    for (int a = 0; a < NU; ++a) dtau[NX + a] = du[a];
    const int ti = i < NT ? i : 0;
    const float di = dtau[ti], zi = z[ti];
    if (p.write_gC) {  // (uniform across the warp; a half without an element stages but never stores)
      float* stg = sh + PC0 + (t & 1) * CBLK;
      if (t >= 2) {
        if (wgc && i == 0) bulk_wait_read<1>();  // the copy of block t - 2 has read this buffer
        __syncwarp();
      }
      // grad_C = -1/2 (dtau (x) z + z (x) dtau), z = [X_t; U_t] (controller.py:87-96)
      if (i < NT) {
        float2* row = reinterpret_cast<float2*>(stg + i * NT);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          const float g0 = -0.5f * (di * z[j] + zi * dtau[j]);
          const float g1 = -0.5f * (di * z[j + 1] + zi * dtau[j + 1]);
          row[j / 2] = make_float2(g0, g1);
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (wgc && i == 0) {
        bulk_store(gCb + (int64_t)t * p.C_tstride * CBLK, stg, CBLK * 4u);
        bulk_commit();
      }
    }
    if (valid && i < NT) {
      if (sigm && p.g_sig != nullptr) {
        float* gq = p.g_sig + b * (int64_t)(2 * NT) * T;
        const float gii = -0.5f * (di * zi + zi * di);
        const int off = sig_off(T, t, i);
        gq[off] = gii * p.sig.range_q;
        const float gc = -di;
        gq[14 * T + off] = i == NX ? (-gc) * p.sig.range_pt : gc * p.sig.range_p;
      }
      if (p.g_c != nullptr) p.g_c[b * p.gc_bstride + t * p.gc_tstride + i] = -di;
      if (i < NX && p.g_xref != nullptr) p.g_xref[(b * (T + 1) + t) * NX + i] = di;
      if (i >= NX && p.g_uref != nullptr) p.g_uref[(b * T + t) * NU + (i - NX)] = di;
    }
    const Jac J = jtab_read(JT + PJT_F * t);
    float nd[NX];
    jac_apply(J, dx, du, nd);
#pragma unroll
    for (int k = 0; k < NX; ++k) dx[k] = nd[k];
  }
  if (wgc && i == 0) bulk_wait<0>();
  __syncwarp();
  if (!valid) return;
  if (p.g_xref != nullptr && i < NX) p.g_xref[(b * (T + 1) + T) * NX + i] = 0.0f;
  if (p.g_Cf != nullptr || p.g_cf != nullptr) {
    float ev[NX];
#pragma unroll
    for (int k = 0; k < NX; ++k)
      ev[k] = ld(Xb, T * NX + k) - (p.x_ref != nullptr ? __ldg(p.x_ref + (b * (T + 1) + T) * NX + k) : 0.0f);
    if (p.g_Cf != nullptr) {
      for (int f = i; f < CBLK; f += HALF) {
        const int r = f / NT, j = f - r * NT;
        float g = 0.0f;
        if (r < NX && j < NX) {
          float dr = 0.0f, dj = 0.0f, er = 0.0f, ej = 0.0f;
#pragma unroll
          for (int q = 0; q < NX; ++q) {
            if (q == r) { dr = dx[q]; er = ev[q]; }
            if (q == j) { dj = dx[q]; ej = ev[q]; }
          }
          g = -0.5f * (dr * ej + er * dj);
        }
        p.g_Cf[b * CBLK + f] = g;
      }
    }
    if (p.g_cf != nullptr && i < NT) p.g_cf[b * NT + i] = i < NX ? -dx[i] : 0.0f;
  }
}

}  // namespace

size_t backward_smem_bytes() { return (size_t)EPW * CBLK * 4 + (size_t)EPW * XS * 4 + sizeof(uint64_t); }

cudaError_t launch_backward(const CUtensorMap& tmC, const CUtensorMap& tmG, const BackwardParams& p,
                            cudaStream_t stream) {
  if (p.T <= PAIR_MAX_T && (p.layout == LAYOUT_PAIR || (p.layout == LAYOUT_AUTO && p.B <= PAIR_MAX_B))) {
    const unsigned pgrid = (unsigned)((p.B + EPWP - 1) / EPWP);
    const size_t psmem = (size_t)EPWP * pair_area(p.T, PREC_F + PJT_F + PKS_F + PLX_F) * sizeof(float);
    const cudaError_t e = allow_smem<backward_pair_kernel<8>>(psmem);
    if (e != cudaSuccess) return e;
    backward_pair_kernel<8><<<pgrid, WARP, psmem, stream>>>(p);
    return cudaGetLastError();
  }
  const size_t smem = backward_smem_bytes();
  const unsigned grid = (unsigned)((p.B + EPW - 1) / EPW);
  const int tier = pick_backward_tier(grid);
  if (tier == TIER_HI) backward_kernel<TIER_HI><<<grid, WARP, smem, stream>>>(tmC, tmG, p);
  else if (tier == TIER_MID) backward_kernel<TIER_MID><<<grid, WARP, smem, stream>>>(tmC, tmG, p);
  else backward_kernel<TIER_LO><<<grid, WARP, smem, stream>>>(tmC, tmG, p);
  return cudaGetLastError();
}

}  // namespace ilqr
