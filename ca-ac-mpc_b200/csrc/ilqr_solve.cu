// ilqr_solve.cu -- fused batched iLQR forward solve (all iterations, one launch).
//
// Mapping: one CTA = one warp = 6 batch elements, a team of 5 lanes per
// element (lanes 30, 31 mirror two lanes of the sixth element). The team splits each Riccati step by rows
// of V (ilqr_team.cuh) and evaluates the line-search step sizes one per lane.
// Per-element state lives in a caller-provided workspace, element-interleaved
// in 16-byte-aligned records (layout in ilqr_kernels.h): SOLVE_SLOTS
// trajectory slots of (x_t, u_t) records, the gains K_t as one float4 per
// state column, k_t, and the diagonals of C_t. The dense cost blocks C[b, t]
// of the warp's six elements are staged into shared memory by one TMA bulk
// tensor copy per step.
//
// Candidate slots: one slot holds the nominal trajectory; the line-search lane
// of step size j (j < SOLVE_SLOTS - 1) stores its candidate rollout into
// another slot as it goes, so accepting candidate j only re-points the
// nominal slot (the stored records are exactly the rollout the reference
// takes as its new X, U). Step sizes beyond those slots (n_alpha > 5) fall
// back to one lane re-running the accepted candidate.
//
// Diagonal cost blocks: the first Riccati pass also checks whether every
// C[b, t] block of the warp's elements is diagonal and copies the diagonals
// into the workspace. If so, later passes stop reading C: the Riccati pass
// rebuilds the blocks in shared memory from the 14 diagonals (off-diagonal
// entries stay exact zeros, so every sum is the one the dense path forms) and
// the line search evaluates tau^T C tau from the diagonals alone. Each product
// with an off-diagonal zero that the dense path adds is an exact zero unless
// tau holds an infinity or NaN, where the dense quadratic form is NaN; the
// diagonal form reproduces that, so results are identical.
//
// Algorithm: DifferentiableMPCController.solve_step (controller.py:303-435)
// with per-element freezing: an element stops at its first non-improving
// iteration, which leaves X, U identical to the reference's global loop.
// The initial objective (controller.py:308) is accumulated during the first
// Riccati pass, which reads the same C_t blocks.
#include "ilqr_kernels.h"
#include "ilqr_pair.cuh"
#include "ilqr_team.cuh"

namespace ilqr {

namespace {

__device__ __forceinline__ float ldg_or0(const float* p, bool ok) { return ok ? __ldg(p) : 0.0f; }

// Line-search staging (the 12-CTA register tier, which has the shared
// memory): per element and step one 368-byte record, copied with
// cp.async one step ahead into one of two buffers: nominal (x, u) at [0, 16),
// k at [16, 20), the ten K columns at [20, 60), the cost record at [60, 92).
constexpr int STG_F = 92;
constexpr int STG_CHUNKS = STG_F / 4;   // 23 copies of 16 bytes
constexpr int STG_OFF = 16;             // bytes between the mbarrier and the first buffer

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

// The workspace records of one element (layout in ilqr_kernels.h). Addresses
// are rebuilt from the kernel parameters on every use (they live in the
// constant bank), so only the element index occupies a register; record
// indices fit in 32 bits (checked by the host).
struct SolveWs {
  const SolveParams& p;
  uint32_t b;
  __device__ __forceinline__ uint32_t S() const { return (uint32_t)p.S; }
  __device__ __forceinline__ float4* rec(int s, int t) const {
    const uint32_t r = ((uint32_t)s * (uint32_t)(p.T + 1) + (uint32_t)t) * S() + b;
    return reinterpret_cast<float4*>(p.ws + (size_t)r * TRJ_REC);
  }
  __device__ __forceinline__ float* gk() const {
    return p.ws + (size_t)SOLVE_SLOTS * (uint32_t)(p.T + 1) * S() * TRJ_REC;
  }
  __device__ __forceinline__ float4* kcol(int t, int j) const {
    const uint32_t r = (uint32_t)(t * NX + j) * S() + b;
    return reinterpret_cast<float4*>(gk() + (size_t)r * 4);
  }
  __device__ __forceinline__ float4* kff(int t) const {
    const uint32_t r = (uint32_t)t * S() + b;
    return reinterpret_cast<float4*>(gk() + (size_t)p.T * NX * S() * 4 + (size_t)r * 4);
  }
  // cost record of step t: diag(C_t) at [0, 14), c_t at [16, 30)
  __device__ __forceinline__ float* diag(int t) const {
    const uint32_t r = (uint32_t)t * S() + b;
    return gk() + (size_t)p.T * (NX + 1) * S() * 4 + (size_t)r * COST_REC;
  }
  __device__ __forceinline__ float* cvec(int t) const { return diag(t) + 16; }
  // segmented solve: the element's saved state, list L's entry pos and
  // list L's count, in floats 12..15 of t = T records (slots 0, 1 + 2 L and
  // 2 + 2 L, the count at element 0)
  __device__ __forceinline__ float4* seg_state() const { return rec(0, p.T) + 3; }
};
__host__ __device__ __forceinline__ int* seg_entry(float* ws, int T, int64_t S, int L, int64_t pos) {
  return reinterpret_cast<int*>(ws + (((size_t)(1 + 2 * L) * (T + 1) + T) * S + pos) * TRJ_REC + 12);
}
__host__ __device__ __forceinline__ int* seg_count(float* ws, int T, int64_t S, int L) {
  return reinterpret_cast<int*>(ws + ((size_t)(2 + 2 * L) * (T + 1) + T) * S * TRJ_REC + 12);
}

__device__ __forceinline__ void load_rec(const float4* r, float (&x)[NX], float (&u)[NU]) {
  const float4 a = r[0], c = r[1], d = r[2], e = r[3];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  x[8] = d.x; x[9] = d.y; u[0] = d.z; u[1] = d.w;
  u[2] = e.x; u[3] = e.y;
}

__device__ __forceinline__ void load_rec_x(const float4* r, float (&x)[NX]) {
  const float4 a = r[0], c = r[1], d = r[2];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  x[8] = d.x; x[9] = d.y;
}

__device__ __forceinline__ void store_rec(float4* r, const float (&x)[NX], const float (&u)[NU]) {
  r[0] = make_float4(x[0], x[1], x[2], x[3]);
  r[1] = make_float4(x[4], x[5], x[6], x[7]);
  r[2] = make_float4(x[8], x[9], u[0], u[1]);
  r[3] = make_float4(u[2], u[3], 0.0f, 0.0f);
}

__device__ __forceinline__ void store_rec_x(float4* r, const float (&x)[NX]) {
  r[0] = make_float4(x[0], x[1], x[2], x[3]);
  r[1] = make_float4(x[4], x[5], x[6], x[7]);
  r[2] = make_float4(x[8], x[9], 0.0f, 0.0f);
}

// torch.clamp semantics: a NaN stays NaN (max.NaN / min.NaN return NaN when
// either operand is NaN; the bounds are finite).
__device__ __forceinline__ float clamp_nan(float v, float lo, float hi) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(v), "f"(lo));
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(r), "f"(hi));
  return r;
}

// Candidate control of the grid line search (controller.py:480-490):
// u = U_t + a k_t + a (K_t (x - X_t)), then max(., u_min), min(., u_max).
// kcol(j) returns column j of K_t (the four gains of state j); each row of
// K_t (x - X_t) is accumulated over j in index order.
// The unclamped candidate ub + (a k + a (K dx)). K dx runs as packed FMA
// chains (controls 0, 1 and 2, 3), in the scalar formula's order; the rest
// stays scalar: a packed multiply whose product feeds a packed add may be
// fused into one packed FMA by the code generator, which rounds once
// instead of twice (measured on B200), so no packed product here ends in an add.
template <class KCol>
__device__ __forceinline__ void candidate_raw(const float (&x)[NX], const float (&xb)[NX], const float (&ub)[NU],
                                              KCol&& kcol, const float (&kt)[NU], float al, float (&v)[NU]) {
  float dx[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) dx[i] = x[i] - xb[i];
  float2 kd01, kd23;
  {
    const float4 c = kcol(0);
    const float2 d = dup2(dx[0]);
    kd01 = mul2(make_float2(c.x, c.y), d);
    kd23 = mul2(make_float2(c.z, c.w), d);
  }
#pragma unroll
  for (int j = 1; j < NX; ++j) {
    const float4 c = kcol(j);
    const float2 d = dup2(dx[j]);
    kd01 = fma2(make_float2(c.x, c.y), d, kd01);
    kd23 = fma2(make_float2(c.z, c.w), d, kd23);
  }
  const float kd[NU] = {kd01.x, kd01.y, kd23.x, kd23.y};
#pragma unroll
  for (int a = 0; a < NU; ++a) v[a] = ub[a] + (al * kt[a] + al * kd[a]);
}

template <class KCol>
__device__ __forceinline__ void candidate_u(const float (&x)[NX], const float (&xb)[NX], const float (&ub)[NU],
                                            KCol&& kcol, const float (&kt)[NU], float al,
                                            const float* __restrict__ lo, const float* __restrict__ hi,
                                            float (&u)[NU]) {
  float v[NU];
  candidate_raw(x, xb, ub, kcol, kt, al, v);
#pragma unroll
  for (int a = 0; a < NU; ++a) u[a] = lo != nullptr ? clamp_nan(v[a], __ldg(lo + a), __ldg(hi + a)) : v[a];
}

// candidate_u with the box in registers (the same operations).
template <class KCol>
__device__ __forceinline__ void candidate_u_reg(const float (&x)[NX], const float (&xb)[NX], const float (&ub)[NU],
                                                KCol&& kcol, const float (&kt)[NU], float al, bool bounds,
                                                const float (&lo)[NU], const float (&hi)[NU], float (&u)[NU]) {
  float v[NU];
  candidate_raw(x, xb, ub, kcol, kt, al, v);
#pragma unroll
  for (int a = 0; a < NU; ++a) u[a] = bounds ? clamp_nan(v[a], lo[a], hi[a]) : v[a];
}

// Whether flat index f (< 196) of a C block is on its diagonal (15 i):
// f / 15 as (f * 2185) >> 15, exact for these f, without a division.
__device__ __forceinline__ bool on_diag(int f) { return f == ((f * 2185) >> 15) * (NT + 1); }

// Whether the four floats at flat indices f .. f + 3 of a C block hold a
// nonzero off the diagonal (bitwise, so that no lane branches).
__device__ __forceinline__ bool offdiag_nonzero(const float4 v, int f) {
  return ((v.x != 0.0f) & !on_diag(f)) | ((v.y != 0.0f) & !on_diag(f + 1)) | ((v.z != 0.0f) & !on_diag(f + 2)) |
         ((v.w != 0.0f) & !on_diag(f + 3));
}

// A lane's share of the scan of one C block for off-diagonal nonzeros: the
// chunks of four floats q0, q0 + stride, ..., a fixed unrolled count with a
// guard, so that lanes with one chunk fewer do not diverge.
template <int STRIDE>
__device__ __forceinline__ bool scan_offdiag(const float* blk, int q0) {
  const float4* c4 = reinterpret_cast<const float4*>(blk);
  bool nz = false;
#pragma unroll
  for (int r = 0; r < (CBLK / 4 + STRIDE - 1) / STRIDE; ++r) {
    const int q = q0 + STRIDE * r;
    const float4 v = c4[q < CBLK / 4 ? q : 0];
    nz |= (q < CBLK / 4) & offdiag_nonzero(v, 4 * q);
  }
  return nz;
}

__device__ __forceinline__ float pick(const float (&v)[NT], int i) {
  float r = v[0];
#pragma unroll
  for (int j = 1; j < NT; ++j) r = (i == j) ? v[j] : r;
  return r;
}

__device__ __forceinline__ float4 f4(const float (&v)[NU]) { return make_float4(v[0], v[1], v[2], v[3]); }

template <int NAC, bool HAS_REF, int MINB>
__global__ void __launch_bounds__(32, MINB) solve_kernel(const __grid_constant__ CUtensorMap tmC,
                                                       const SolveParams p) {
  static_assert(NAC == TEAM, "one step size per team lane");
  // Staging pays at the 12-CTA tier (B=8192: -9 %), which stages the whole
  // record; the 19-CTA tier has shared memory for the K columns only. At 8
  // CTAs per SM the loads are short already and the copies cost more than
  // they hide.
  constexpr bool STAGE = MINB != TIER_HI;
  constexpr bool FULL_REC = MINB == TIER_MID;
  constexpr int SF = FULL_REC ? STG_F : 40;       // floats per element and buffer
  constexpr int Q0 = FULL_REC ? 0 : 5;            // first chunk of the record staged
  constexpr int NQ = FULL_REC ? STG_CHUNKS : 10;  // chunks staged
  static_assert(NAC <= SOLVE_SLOTS - 1, "a slot per candidate of the first chunk");
  extern __shared__ __align__(128) unsigned char smem[];
  float* slab = reinterpret_cast<float*>(smem);
  float* xch = slab + EPW * CBLK;
  uint64_t* bar = reinterpret_cast<uint64_t*>(xch + EPW * XS);
  const int lane = threadIdx.x;
  // Lanes 30, 31 mirror lanes 25, 26 (element 5, members 0 and 1): they load
  // and compute exactly what those lanes do, so their shared-memory writes are
  // bit-identical to the ones they duplicate, and they write no global memory.
  const bool dup = lane >= EPW * TEAM;
  const int e = dup ? EPW - 1 : lane / TEAM;
  const int m = lane - (dup ? EPW * TEAM : e * TEAM);
  const int base = e * TEAM;
  const int64_t b0 = (int64_t)blockIdx.x * EPW;
  const bool resume = p.seg_in >= 0;
  int64_t b = b0 + e;
  bool valid = b < p.B;  // the lane's element exists (loads, compute)
  if (resume) {          // elements from the list the previous launch made
    int64_t cnt = *(volatile const int*)seg_count(p.ws, p.T, p.S, p.seg_in);
    cnt = cnt < 0 ? 0 : (cnt > p.B ? p.B : cnt);
    if (b0 >= cnt) return;  // the whole CTA lies beyond the list
    valid = b < cnt;
    const int64_t ent = valid ? (int64_t)*seg_entry(p.ws, p.T, p.S, p.seg_in, b) : 0;
    valid = valid && ent >= 0 && ent < p.B;  // (an entry out of range is skipped)
    b = valid ? ent : 0;
  }
  const bool own = valid && !dup;  // ... and this lane writes its results
  const int64_t bw = valid ? b : (resume ? 0 : b0);  // workspace record read by this lane (never written when !own)
  const int T = p.T;
  const float dt = p.dt;
  const SolveWs W{p, (uint32_t)bw};

  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  TeamPipe pipe{slab, bar, 0u, &tmC, (int)b0, true};
  float* xc = xch + e * XS;
  float* Ce = slab + e * CBLK;
  const int ra = row_a(m), rb = row_b(m);

  const bool bounds = p.has_bounds != 0;
  const float* lo = bounds ? p.u_min : nullptr;
  const float* hi = bounds ? p.u_max : nullptr;
  const float* cb = p.c != nullptr ? p.c + b * p.c_bstride : nullptr;
  const float* xrb = (HAS_REF && p.x_ref != nullptr) ? p.x_ref + b * (int64_t)(T + 1) * NX : nullptr;
  const float* urb = (HAS_REF && p.u_ref != nullptr) ? p.u_ref + b * (int64_t)T * NU : nullptr;
  auto xref = [&](int t, int i) { return (HAS_REF && xrb != nullptr) ? ldg_or0(xrb + t * NX + i, valid) : 0.0f; };
  auto uref = [&](int t, int a) { return (HAS_REF && urb != nullptr) ? ldg_or0(urb + t * NU + a, valid) : 0.0f; };
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;
  const float* cf = (p.c_f != nullptr && valid) ? p.c_f + b * NT : nullptr;
  // staging buffers of this element (STAGE only): buffer s at stg + s * EPW * STG_F
  float* stg = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(bar) + STG_OFF) + e * SF;

  auto load_x0 = [&](float (&x)[NX]) {
#pragma unroll
    for (int i = 0; i < NX; ++i) x[i] = ldg_or0(p.x0 + b * NX + i, valid);
  };
  const bool writer = own && m == 0;
  if (p.trace != nullptr && writer && !resume)
    for (int i = 0; i < p.max_iter; ++i) p.trace[b * p.max_iter + i] = (int8_t)-128;

  // ---- initial open-loop rollout with U_init into slot 0 (controller.py:305, 578-603)
  if (!resume) {
    float x[NX];
    load_x0(x);
    for (int t = 0; t < T; ++t) {
      float u[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) u[a] = ldg_or0(p.U_init + (b * T + t) * NU + a, valid);
      if (writer) store_rec(W.rec(0, t), x, u);
      float xn[NX];
      drone_step(x, u, dt, xn);
#pragma unroll
      for (int i = 0; i < NX; ++i) x[i] = xn[i];
    }
    if (writer) store_rec_x(W.rec(0, T), x);
  }
  __syncwarp();

  int nom = 0;  // slot of the nominal trajectory (the same in every lane of a team)
  auto stage_ls = [&](int t, int buf) {  // issue the copies of step t's record (the owner lanes of a team)
    if (!dup) {
      float* d = stg + buf * EPW * SF;
#pragma unroll
      for (int i = 0; i < (NQ + TEAM - 1) / TEAM; ++i) {
        const int q = Q0 + m + TEAM * i;
        if (q < Q0 + NQ) {
          const void* src = q < 4    ? (const void*)(W.rec(nom, t) + q)
                            : q == 4 ? (const void*)W.kff(t)
                            : q < 15 ? (const void*)W.kcol(t, q - 5)
                                     : (const void*)(W.diag(t) + 4 * (q - 15));
          cp_async16(d + 4 * (q - Q0), src);
        }
      }
    }
    cp_async_commit();
  };
  uint32_t status = 0;
  bool active = valid;
  int iters = 0;
  int stall_iter = p.max_iter;
  float stall_gap = 0.0f;
  float best = 0.0f;
  // Costs from policy parameters are diagonal by construction: the slab holds
  // zeros off the diagonal from the start, and no pass reads C.
  const bool sigm = p.sig.p != nullptr;
  const float* sgrow = sigm ? p.sig.p + bw * (int64_t)(2 * NT) * T : nullptr;
  // warp-uniform: all C[b, t] of the warp's elements are diagonal (known
  // after pass 1; every resumed element comes from such a warp)
  bool diag = sigm || resume;
  bool offd = false;  // this lane saw a nonzero off-diagonal entry during pass 1
  if (diag) {
    for (int f = lane; f < EPW * CBLK; f += WARP) slab[f] = 0.0f;
    __syncwarp();
  }
  // resumed launch: every lane starts at iteration seg_it0 (warp-uniform); a
  // listed element restores the state the previous launch saved (it improved
  // in every iteration so far). Lanes past the end of the list keep slot 0
  // of their stand-in element: its saved state may never have been written.
  const int it_begin = resume ? p.seg_it0 : 0;
  if (resume && valid) {
    const float4 st = *W.seg_state();
    nom = __float_as_int(st.x);
    nom = nom < 0 ? 0 : (nom >= SOLVE_SLOTS ? SOLVE_SLOTS - 1 : nom);
    best = st.y;
    status = __float_as_uint(st.z);
    iters = p.seg_it0;
  }
  bool deferred = false;  // this element continues in the next launch

  // The first pass always runs: it also yields the initial objective (with
  // max_iter == 0 only that).
  const int n_loop = p.max_iter > 0 ? p.max_iter : 1;
  for (int it = it_begin; it < n_loop; ++it) {
    const bool cost_only = it >= p.max_iter;
    if (!cost_only && p.forced != nullptr && active && p.forced[b * p.max_iter + it] == (int8_t)-128)
      active = false;
    if (!__any_sync(FULL, active) && it > 0) break;

    // ---- backward Riccati pass (controller.py:315-318, 697-723) ------------
    float Va[NX], Vb[NX], va_, vb_;
    {
      float xT[NX], tn[NX];
      load_rec_x(W.rec(nom, T), xT);
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = xT[i] - xref(T, i);
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
    auto ric_body = [&](int t, auto&& next) {
      float xb[NX], ub[NU], tau[NT];
      // every global load of the step is issued here, before the first use
      load_rec(W.rec(nom, t), xb, ub);
      const int ru = NX + (m < NU ? m : 0);
      // c_t from the input on the first pass (which copies it into the cost
      // record), from the record afterwards
      float ca_, cb_, cu;
      if (first && sigm) {
        ca_ = sig_c(p.sig, sgrow, T, t, ra);
        cb_ = sig_c(p.sig, sgrow, T, t, rb);
        cu = sig_c(p.sig, sgrow, T, t, ru);
      } else if (first) {
        ca_ = ldg_or0(cb + t * p.c_tstride + ra, valid);
        cb_ = ldg_or0(cb + t * p.c_tstride + rb, valid);
        cu = ldg_or0(cb + t * p.c_tstride + ru, valid);
      } else {
        const float* cr = W.cvec(t);
        ca_ = cr[ra];
        cb_ = cr[rb];
        cu = cr[ru];
      }
      if (diag && first && sigm) {  // build the diagonal from the parameters, keep a copy
        float* dgt = W.diag(t);
#pragma unroll
        for (int s3 = 0; s3 < 3; ++s3) {
          const int i = m + TEAM * s3;
          if (i < NT) {
            const float dv = sig_diag(p.sig, sgrow, T, t, i);
            Ce[i * (NT + 1)] = dv;
            if (own) dgt[i] = dv;
          }
        }
        __syncwarp();
      } else if (diag) {  // rebuild the diagonal of the slab from the workspace copy
        const float* dgt = W.diag(t);
#pragma unroll
        for (int s3 = 0; s3 < 3; ++s3)
          if (m + TEAM * s3 < NT) Ce[(m + TEAM * s3) * (NT + 1)] = dgt[m + TEAM * s3];
        __syncwarp();
      }
#pragma unroll
      for (int i = 0; i < NX; ++i) tau[i] = xb[i] - xref(t, i);
#pragma unroll
      for (int a = 0; a < NU; ++a) tau[NX + a] = ub[a] - uref(t, a);
      // quadraticize my rows (cost.py:149-165): l_tau = C tau + c
      auto rowdot = [&](int r) {
        const float* Cr = Ce + r * NT;
        float s = Cr[0] * tau[0];
#pragma unroll
        for (int j = 1; j < NT; ++j) s = fmaf(Cr[j], tau[j], s);
        return s;
      };
      const float sa = rowdot(ra), sb = rowdot(rb);
      const float lxa = sa + ca_, lxb = sb + cb_;
      const float su = rowdot(ru);
      if (m < NU) xc[X_LU + m] = su + cu;
      if (first) {
        if (own) {
          float* cr = W.cvec(t);
          cr[ra] = ca_;
          cr[rb] = cb_;
          if (m < NU) cr[ru] = cu;
        }
        const float ta = pick(tau, ra), tb = pick(tau, rb), tu = pick(tau, ru);
        cost_q += fmaf(ta, sa, tb * sb) + (m < NU ? tu * su : 0.0f);
        cost_l += fmaf(ca_, ta, cb_ * tb) + (m < NU ? cu * tu : 0.0f);
        if (p.diag_cache && valid && !sigm) {  // (mirror lanes check too; only owners write)
          // the team scans the block for off-diagonal nonzeros (the diagonal
          // sits at flat index 15 i) and keeps a copy of the diagonal
          offd |= scan_offdiag<TEAM>(Ce, m);
          float* dgt = W.diag(t);
#pragma unroll
          for (int s3 = 0; s3 < 3; ++s3)
            if (own && m + TEAM * s3 < NT) dgt[m + TEAM * s3] = Ce[(m + TEAM * s3) * (NT + 1)];
        }
      }
      __syncwarp();
      const Jac J = drone_jac(xb, ub, dt);
      float Ka[NU], Kb[NU], k[NU];
      if (!team_riccati<false, (MINB < TIER_LO)>(Va, Vb, va_, vb_, J, DenseC{Ce}, lxa, lxb, p.reg, 0u, m, valid, xc,
                                                 next, Ka, Kb, k))
        fallback = true;
      if (own) {
        *W.kcol(t, ra) = f4(Ka);
        *W.kcol(t, rb) = f4(Kb);
        if (m == 0) *W.kff(t) = f4(k);
      }
    };
    bool ok = pipe.run(T, true, !diag, [](int) {}, ric_body);
    if (!ok) {
      status |= ELEM_PIPE_TIMEOUT;
      active = false;
      break;
    }
    if (first && p.diag_cache && !sigm) {
      diag = !__any_sync(FULL, offd);
      if (diag) {  // off-diagonal entries of the rebuilt blocks stay zero from here on
        for (int f = lane; f < EPW * CBLK; f += WARP) slab[f] = 0.0f;
        __syncwarp();
      }
    }
    if (team_sum(fallback ? 1.0f : 0.0f, base) > 0.0f && active) status |= ELEM_CHOL_FALLBACK;
    if (first) {
      float xT[NX], tn[NX];
      load_rec_x(W.rec(nom, T), xT);
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = xT[i] - xref(T, i);
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
      const int j = a0 + m;
      const float al = (j < p.n_alpha) ? p.alphas[j] : 0.0f;
      const bool keep = own && j < p.n_alpha && j < SOLVE_SLOTS - 1;  // candidate stored in a slot
      const int cs = j < nom ? j : j + 1;
      float x[NX], sq = 0.0f, sl = 0.0f;
      load_x0(x);
      auto ls_body = [&](int t, auto&& next) {
        float xb[NX], ub[NU], kt[NU], u[NU];
        // step t's record: staged one step ahead (STAGE) or read directly
        const float* sb = stg + (t & 1) * EPW * SF;  // staged chunks Q0.. of step t's record
        if constexpr (STAGE) {
          if (t + 1 < T) {
            stage_ls(t + 1, (t + 1) & 1);
            cp_async_wait<1>();
          } else {
            cp_async_wait<0>();
          }
          __syncwarp();
        }
        const float4* rec_t = FULL_REC ? reinterpret_cast<const float4*>(sb) : W.rec(nom, t);
        const float4* kff_t = FULL_REC ? reinterpret_cast<const float4*>(sb + 16) : W.kff(t);
        const float4* kcol_t = STAGE ? reinterpret_cast<const float4*>(sb + 20 - 4 * Q0) : W.kcol(t, 0);
        const float* cost_t = FULL_REC ? sb + 60 : W.diag(t);
        const int64_t kstride = STAGE ? 1 : (int64_t)p.S;  // float4s between K columns
        load_rec(rec_t, xb, ub);
        {
          const float4 k4 = *kff_t;
          kt[0] = k4.x; kt[1] = k4.y; kt[2] = k4.z; kt[3] = k4.w;
        }
        candidate_u(x, xb, ub, [&](int jj) { return kcol_t[jj * kstride]; }, kt, al, lo, hi, u);
        if (keep) store_rec(W.rec(cs, t), x, u);
        float tau[NT];
#pragma unroll
        for (int i = 0; i < NX; ++i) tau[i] = x[i] - xref(t, i);
#pragma unroll
        for (int a = 0; a < NU; ++a) tau[NX + a] = u[a] - uref(t, a);
        float l;  // c^T tau, c_t from the cost record
        {
          const float4* c4 = reinterpret_cast<const float4*>(cost_t + 16);
          const float4 h0 = c4[0], h1 = c4[1], h2 = c4[2], h3 = c4[3];
          const float cv[NT] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z,
                                h1.w, h2.x, h2.y, h2.z, h2.w, h3.x, h3.y};
          l = cv[0] * tau[0];
#pragma unroll
          for (int jj = 1; jj < NT; ++jj) l = fmaf(cv[jj], tau[jj], l);
        }
        float q = 0.0f;
        if (diag) {
          const float4* d4 = reinterpret_cast<const float4*>(cost_t);
          const float4 g0 = d4[0], g1 = d4[1], g2 = d4[2], g3 = d4[3];
          const float dgv[NT] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z,
                                 g1.w, g2.x, g2.y, g2.z, g2.w, g3.x, g3.y};
#pragma unroll
          for (int i = 0; i < NT; ++i) q = fmaf(tau[i], dgv[i] * tau[i], q);
          // The dense form is NaN when any tau_j is infinite or NaN (an
          // off-diagonal 0 times it); the diagonal sum is then not finite
          // either, so only a non-finite q needs the check.
          if (!isfinite(q)) {
            bool nonfinite = false;
#pragma unroll
            for (int i = 0; i < NT; ++i) nonfinite |= !isfinite(tau[i]);
            if (nonfinite) q = __int_as_float(0x7fffffff);
          }
        } else {
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            const float2* r2 = reinterpret_cast<const float2*>(Ce + i * NT);
            float r = 0.0f;
#pragma unroll
            for (int jj = 0; jj < NT / 2; ++jj) {
              const float2 c2 = r2[jj];
              r = (jj == 0) ? c2.x * tau[0] : fmaf(c2.x, tau[2 * jj], r);
              r = fmaf(c2.y, tau[2 * jj + 1], r);
            }
            q = fmaf(tau[i], r, q);
          }
        }
        next();
        sq += q;
        sl += l;
        float xn[NX];
        drone_step(x, u, dt, xn);
#pragma unroll
        for (int i = 0; i < NX; ++i) x[i] = xn[i];
      };
      if constexpr (STAGE) stage_ls(0, 0);
      ok = pipe.run(T, false, !diag, [](int) {}, ls_body);
      if (!ok) break;
      if (keep) store_rec_x(W.rec(cs, T), x);
      float tn[NX];
#pragma unroll
      for (int i = 0; i < NX; ++i) tn[i] = x[i] - xref(T, i);
      const float mine = (0.5f * sq + sl) + terminal_cost(Cf, cf, tn);
      // gather the team's costs; torch.argmin semantics (first NaN, else first minimum)
#pragma unroll
      for (int jj = 0; jj < NAC; ++jj) {
        const float cj = __shfl_sync(FULL, mine, (base + jj) & 31);
        if (a0 + jj >= p.n_alpha) continue;
        cand[a0 + jj] = cj;
        if (!nan_seen) {
          if (cj != cj) {
            nan_seen = true;
            jbest = a0 + jj;
            cmin = cj;
          } else if (!have || cj < cmin) {
            have = true;
            jbest = a0 + jj;
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
      if (p.trace != nullptr && m == 0 && own) p.trace[b * p.max_iter + it] = (int8_t)(accept ? jsel : -(jbest + 1));
      if (!accept && stall_iter == p.max_iter) {
        stall_iter = it;
        stall_gap = fabsf(cmin - best);
      }
      if (accept) best = cand[jsel];
      if (!accept && p.forced == nullptr) active = false;
    }
    // ---- new nominal: the accepted candidate's slot, or a re-run into a free
    // slot for a step size that had none --------------------------------------
    const bool rerun = accept && jsel >= SOLVE_SLOTS - 1;
    if (accept && !rerun) nom = jsel < nom ? jsel : jsel + 1;
    if (__any_sync(FULL, rerun)) {
      const int dst = nom == 0 ? 1 : 0;
      if (rerun && m == 0 && own) {
        const float al = p.alphas[jsel];
        float x[NX];
        load_x0(x);
        for (int t = 0; t < T; ++t) {
          float xb[NX], ub[NU], kt[NU], u[NU];
          load_rec(W.rec(nom, t), xb, ub);
          const float4 k4 = *W.kff(t);
          kt[0] = k4.x; kt[1] = k4.y; kt[2] = k4.z; kt[3] = k4.w;
          candidate_u(x, xb, ub, [&](int jj) { return *W.kcol(t, jj); }, kt, al, lo, hi, u);
          store_rec(W.rec(dst, t), x, u);
          float xn[NX];
          drone_step(x, u, dt, xn);
#pragma unroll
          for (int i = 0; i < NX; ++i) x[i] = xn[i];
        }
        store_rec_x(W.rec(dst, T), x);
      }
      if (rerun) nom = dst;
      __syncwarp();
    }
    if (p.seg_out >= 0 && it + 1 == p.seg_it1 && diag) {
      // Elements still improving continue in the next launch, six per warp;
      // this warp stops here.
      deferred = active;
      if (deferred && writer) {
        *W.seg_state() = make_float4(__int_as_float(nom), best, __uint_as_float(status), 0.0f);
        const int pos = atomicAdd(seg_count(p.ws, p.T, p.S, p.seg_out), 1);
        *seg_entry(p.ws, p.T, p.S, p.seg_out, pos) = (int)b;
      }
      break;
    }
  }

  // ---- outputs (lanes of a team split the writes) -----------------------------
  bool finite = true;
  if (own && !deferred) {
    const float* nrec = reinterpret_cast<const float*>(W.rec(nom, 0));
    const int64_t rstride = p.S * TRJ_REC;  // floats between the records of t and t + 1
    for (int f = m; f < (T + 1) * NX; f += TEAM) {
      const int t = f / NX, i = f - t * NX;
      const float xv = nrec[t * rstride + i];
      finite &= isfinite(xv);
      p.X[b * (T + 1) * NX + f] = xv;
    }
    for (int f = m; f < T * NU; f += TEAM) {
      const int t = f / NU, a = f - t * NU;
      const float uv = nrec[t * rstride + NX + a];
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
  if (diag) status |= ELEM_DIAG_COST;
  if (writer && !deferred) {
    if (p.iters) p.iters[b] = iters;
    if (p.status) p.status[b] = status;
    if (p.best_cost) p.best_cost[b] = best;
    if (p.stall_iter) p.stall_iter[b] = stall_iter;
    if (p.stall_gap) p.stall_gap[b] = stall_gap;
  }
}


// The pair layout of the same solve (ilqr_pair.cuh): one element per
// half-warp. Lane i < 10 owns row i of V through the Riccati pass; the line
// search runs step size j on lane j of the half (up to eight at once); C_t
// blocks stream through a cp.async double buffer. Workspace records, the
// candidate slots and every formula are the team kernel's, so the results
// are the same bits.
//
// Per-step tables in shared memory keep the serial chain of each step short:
// at the start of every Riccati pass the sixteen lanes load the nominal
// records of all steps and evaluate all the Jacobians at once (drone_jac into
// a Jacobian table, one step per lane and round); the pass then reads its
// step's record and Jacobian from shared memory and each lane picks its row
// coefficients from the table by offsets fixed at kernel start. The pass
// also leaves the gains and the cost records of every step in shared memory,
// so the line search that follows loads nothing from global memory but the
// dense cost blocks.
template <bool HAS_REF, int MINB>
__global__ void __launch_bounds__(32, MINB) solve_pair_kernel(const SolveParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x;
  const int h = lane >> 4, i = lane & (HALF - 1);
  const int base = h * HALF;
  const int64_t b0 = (int64_t)blockIdx.x * EPWP;
  const int64_t b = b0 + h;
  const bool valid = b < p.B;
  const int64_t bw = valid ? b : b0;  // workspace record read by this half (never written when !valid)
  const int T = p.T;
  const float dt = p.dt;
  const SolveWs W{p, (uint32_t)bw};
  float* sh = reinterpret_cast<float*>(smem) + h * pair_area(T, PREC_F + PJT_F + PKS_F + PCR_F, CBLK);
  float* REC = sh + PBASE;                  // [T][16] nominal x_t, u_t
  float* JT = REC + PREC_F * T;             // [T][32] Jacobian tables
  float* KS = JT + PJT_F * T;               // [T][44] K columns (4 each), then k
  float* CR = KS + PKS_F * T;               // [T][32] diag(C_t) at 0, c_t at 16
  int own;
  const uint64_t coffs = pair_coef_offsets(i < NT ? i : NT - 1, own);

  const bool bounds = p.has_bounds != 0;
  const float* lo = bounds ? p.u_min : nullptr;
  const float* hi = bounds ? p.u_max : nullptr;
  float blo[NU], bhi[NU];  // the box, in registers for the line search
#pragma unroll
  for (int a = 0; a < NU; ++a) {
    blo[a] = bounds ? __ldg(lo + a) : 0.0f;
    bhi[a] = bounds ? __ldg(hi + a) : 0.0f;
  }
  const float* cb = p.c != nullptr ? p.c + b * p.c_bstride : nullptr;
  const float* xrb = (HAS_REF && p.x_ref != nullptr) ? p.x_ref + b * (int64_t)(T + 1) * NX : nullptr;
  const float* urb = (HAS_REF && p.u_ref != nullptr) ? p.u_ref + b * (int64_t)T * NU : nullptr;
  auto xref = [&](int t, int k) { return (HAS_REF && xrb != nullptr) ? ldg_or0(xrb + t * NX + k, valid) : 0.0f; };
  auto uref = [&](int t, int a) { return (HAS_REF && urb != nullptr) ? ldg_or0(urb + t * NU + a, valid) : 0.0f; };
  const float* Cf = (p.C_f != nullptr && valid) ? p.C_f + b * CBLK : nullptr;
  const float* cf = (p.c_f != nullptr && valid) ? p.c_f + b * NT : nullptr;
  auto load_x0 = [&](float (&x)[NX]) {
#pragma unroll
    for (int k = 0; k < NX; ++k) x[k] = ldg_or0(p.x0 + b * NX + k, valid);
  };
  const bool writer = valid && i == 0;
  if (p.trace != nullptr && writer)
    for (int it = 0; it < p.max_iter; ++it) p.trace[b * p.max_iter + it] = (int8_t)-128;

  const bool sigm = p.sig.p != nullptr;
  const float* sgrow = sigm ? p.sig.p + bw * (int64_t)(2 * NT) * T : nullptr;
  // U_init of every step into the record table (a step per lane), then c_t
  // of every step into the cost records (all (t, k) at once), as cp.async
  // groups in that order: the rollout below waits for the first only, and
  // the second completes behind it. From policy parameters the cost records
  // (c_t and diag C_t) are computed instead.
  for (int t = i; t < T; t += HALF) {
    float* r = REC + PREC_F * t;
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      if (valid) cp_async_f32(r + NX + a, p.U_init + (b * T + t) * NU + a);
      else r[NX + a] = 0.0f;
    }
  }
  cp_async_commit();
  if (sigm) {
#pragma unroll 4
    for (int f = i; f < T * NT; f += HALF) {
      const int t = f / NT, k = f - t * NT;
      float* cr = CR + PCR_F * t;
      cr[16 + k] = sig_c(p.sig, sgrow, T, t, k);
      cr[k] = sig_diag(p.sig, sgrow, T, t, k);
    }
  } else {
    for (int f = i; f < T * NT; f += HALF) {
      const int t = f / NT, k = f - t * NT;
      float* d = CR + PCR_F * t + 16 + k;
      if (valid) cp_async_f32(d, cb + t * p.c_tstride + k);
      else *d = 0.0f;
    }
  }
  cp_async_commit();

  // ---- initial open-loop rollout with U_init into slot 0 (and the record table)
  {
    cp_async_wait<1>();  // this lane's U_init copies
    __syncwarp();
    float x[NX];
    load_x0(x);
    for (int t = 0; t < T; ++t) {
      float u[NU];
#pragma unroll
      for (int a = 0; a < NU; ++a) u[a] = REC[PREC_F * t + NX + a];
      if (writer) store_rec(W.rec(0, t), x, u);
      if (i == 0) store_rec(reinterpret_cast<float4*>(REC + PREC_F * t), x, u);
      float xn[NX];
      drone_step(x, u, dt, xn);
#pragma unroll
      for (int k = 0; k < NX; ++k) x[k] = xn[k];
    }
    if (writer) store_rec_x(W.rec(0, T), x);
  }
  cp_async_wait<0>();  // this lane's cost-record copies
  __syncwarp();

  PairCPipe cpipe{sigm ? nullptr : p.C + bw * p.C_bstride * CBLK, p.C_tstride, sh + PC0, i,
                  sh + PBASE + (PREC_F + PJT_F + PKS_F + PCR_F) * T};
  bool diag = sigm;
  bool offd = false;
  if (sigm) {
    for (int f = i; f < CBLK; f += HALF) sh[PC0 + f] = 0.0f;
    __syncwarp();
  }
  int nom = 0;
  uint32_t status = 0;
  bool active = valid;
  int iters = 0;
  int stall_iter = p.max_iter;
  float stall_gap = 0.0f;
  float best = 0.0f;
  const int ri = i < NX ? i : 0;  // V row of this lane (lanes >= 10 carry a copy of row 0, unused)
  const int ti = i < NT ? i : 0;  // tau / c entry of this lane

  const int n_loop = p.max_iter > 0 ? p.max_iter : 1;
  for (int it = 0; it < n_loop; ++it) {
    const bool cost_only = it >= p.max_iter;
    if (!cost_only && p.forced != nullptr && active && p.forced[b * p.max_iter + it] == (int8_t)-128)
      active = false;
    if (!__any_sync(FULL, active) && it > 0) break;

    // ---- backward Riccati pass ----------------------------------------------------
    float Vr[NX], vr;
    {
      float xT[NX], tn[NX];
      load_rec_x(W.rec(nom, T), xT);
#pragma unroll
      for (int k = 0; k < NX; ++k) tn[k] = xT[k] - xref(T, k);
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < NX; ++j) {
        Vr[j] = Cf ? __ldg(Cf + ri * NT + j) : 0.0f;
        acc = fmaf(Vr[j], tn[j], acc);
      }
      vr = acc + (cf ? __ldg(cf + ri) : 0.0f);
    }
    bool fallback = false;
    float cost_q = 0.0f, cost_l = 0.0f;
    const bool first = (it == 0);
    if (!diag) {  // two blocks in flight ahead of the step that works on a third
      cpipe.issue(T - 1);
      if (T >= 2) cpipe.issue(T - 2);
    }
    // prologue: every step's nominal record (already in the table on the
    // first pass: the initial rollout wrote it) and Jacobian table, a step per lane
    for (int t = i; t < T; t += HALF) {
      float xb[NX], ub[NU];
      float4* d4 = reinterpret_cast<float4*>(REC + PREC_F * t);
      if (!first) {
        const float4* r4 = W.rec(nom, t);
        const float4 q0 = r4[0], q1 = r4[1], q2 = r4[2], q3 = r4[3];
        d4[0] = q0; d4[1] = q1; d4[2] = q2; d4[3] = q3;
      }
      load_rec(reinterpret_cast<const float4*>(d4), xb, ub);
      jtab_write(JT + PJT_F * t, drone_jac(xb, ub, dt));
    }
    __syncwarp();
    for (int t = T - 1; t >= 0; --t) {
      // the step's Jacobian, row coefficients and record (tables written by
      // the prologue, read-only during the pass)
      const float* jt = JT + PJT_F * t;
      const Jac J = jtab_read(jt);
      float cf_[7], c7;
      pair_coef_load(jt, coffs, cf_, c7);
      float xb[NX], ub[NU], tau[NT];
      load_rec(reinterpret_cast<const float4*>(REC + PREC_F * t), xb, ub);
      float* cr = CR + PCR_F * t;
      const float cv = cr[16 + ti];  // c_t entry ti
      if (!diag) {
        if (t >= 2) {
          cpipe.issue(t - 2);
          cp_async_wait<2>();
        } else if (t == 1) {
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
      } else {
        if (i < NT) sh[PC0 + i * (NT + 1)] = cr[i];
      }
      __syncwarp();
      const float* Ce = diag ? sh + PC0 : cpipe.block(t);
#pragma unroll
      for (int k = 0; k < NX; ++k) tau[k] = xb[k] - xref(t, k);
#pragma unroll
      for (int a = 0; a < NU; ++a) tau[NX + a] = ub[a] - uref(t, a);
      // quadraticize: l_tau = C tau + c, row ti (inside the Riccati step,
      // where its chain overlaps the rows of V A)
      float sdot;
      auto lx_fn = [&]() {
        const float2* Cr = reinterpret_cast<const float2*>(Ce + ti * NT);
        float2 c2 = Cr[0];
        float s_ = c2.x * tau[0];
        s_ = fmaf(c2.y, tau[1], s_);
#pragma unroll
        for (int j = 1; j < NT / 2; ++j) {
          c2 = Cr[j];
          s_ = fmaf(c2.x, tau[2 * j], s_);
          s_ = fmaf(c2.y, tau[2 * j + 1], s_);
        }
        sdot = s_;
        return s_ + cv;
      };
      float Kr[NU];
      if (!pair_riccati<false>(Vr, vr, J, cf_, c7, own, Ce, lx_fn, p.reg, 0u, i, valid, sh, Kr)) fallback = true;
      if (i <= NX) *reinterpret_cast<float4*>(KS + PKS_F * t + 4 * i) = f4(Kr);
      if (first) {
        // C_t's buffer is intact until the next step issues its copy
        if (i < NT) {
          sh[PS + i] = sdot;
          sh[PCV + i] = cv;
        }
        if (!sigm) {
          if (i < NT) cr[i] = Ce[i * (NT + 1)];
          if (p.diag_cache && valid) {
            offd |= scan_offdiag<HALF>(Ce, i);
          }
        }
        __syncwarp();
        if (i < TEAM) {
          // the initial objective, accumulated as the team kernel's lane m = i does
          const int ra = row_a(i), rb = row_b(i), ru = NX + (i < NU ? i : 0);
          float xr[NX], ur[NU];
          load_rec(reinterpret_cast<const float4*>(REC + PREC_F * t), xr, ur);
          const float ta = xr[ra] - xref(t, ra), tb = xr[rb] - xref(t, rb), tu = ur[ru - NX] - uref(t, ru - NX);
          const float sa = sh[PS + ra], sb = sh[PS + rb], su = sh[PS + ru];
          const float ca_ = sh[PCV + ra], cb_ = sh[PCV + rb], cu = sh[PCV + ru];
          cost_q += fmaf(ta, sa, tb * sb) + (i < NU ? tu * su : 0.0f);
          cost_l += fmaf(ca_, ta, cb_ * tb) + (i < NU ? cu * tu : 0.0f);
        }
        __syncwarp();
      }
    }
    if (first && p.diag_cache && !sigm) {
      diag = !__any_sync(FULL, offd);
      if (diag) {  // off-diagonal entries of the rebuilt block stay zero from here on
        for (int f = i; f < CBLK; f += HALF) sh[PC0 + f] = 0.0f;
        __syncwarp();
      }
    }
    if (fallback && active) status |= ELEM_CHOL_FALLBACK;
    if (first) {
      float xT[NX], tn[NX];
      load_rec_x(W.rec(nom, T), xT);
#pragma unroll
      for (int k = 0; k < NX; ++k) tn[k] = xT[k] - xref(T, k);
      best = (0.5f * pair_sum5(cost_q, base) + pair_sum5(cost_l, base)) + terminal_cost(Cf, cf, tn);
    }
    __syncwarp();
    if (cost_only) break;

    // ---- grid line search: lane j of the half = step size j ----------------------
    int jbest = 0;
    float cmin = 0.0f;
    bool have = false, nan_seen = false;
    float cand[ILQR_MAX_ALPHAS_DEV];
    {
      const int j = i;
      const float al = (j < p.n_alpha) ? p.alphas[j] : 0.0f;
      const bool keep = valid && j < p.n_alpha && j < SOLVE_SLOTS - 1;
      const int cs = j < nom ? j : j + 1;
      float x[NX], sq = 0.0f, sl = 0.0f;
      load_x0(x);
      // Step cost l = c_t . tau and q = sum_k tau_k (diag(C_t)_k tau_k) of
      // one step from its cost record (diagonal costs); a non-finite q with a
      // non-finite tau becomes NaN (the dense form's 0 * inf), as in the
      // dense-cost loop below.
      auto diag_cost = [&](const float (&tau)[NT], int t, float& l, float& q) {
        const float* cost_t = CR + PCR_F * t;
        const float4* c4 = reinterpret_cast<const float4*>(cost_t + 16);
        const float4 h0 = c4[0], h1 = c4[1], h2 = c4[2], h3 = c4[3];
        const float cvv[NT] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z,
                               h1.w, h2.x, h2.y, h2.z, h2.w, h3.x, h3.y};
        l = cvv[0] * tau[0];
#pragma unroll
        for (int jj = 1; jj < NT; ++jj) l = fmaf(cvv[jj], tau[jj], l);
        const float4* d4 = reinterpret_cast<const float4*>(cost_t);
        const float4 g0 = d4[0], g1 = d4[1], g2 = d4[2], g3 = d4[3];
        const float dgv[NT] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z,
                               g1.w, g2.x, g2.y, g2.z, g2.w, g3.x, g3.y};
        q = 0.0f;
#pragma unroll
        for (int k = 0; k < NT; ++k) q = fmaf(tau[k], dgv[k] * tau[k], q);
      };
      auto nan_fix = [](const float (&tau)[NT], float& q) {
        if (!isfinite(q)) {
          bool nonfinite = false;
#pragma unroll
          for (int k = 0; k < NT; ++k) nonfinite |= !isfinite(tau[k]);
          if (nonfinite) q = __int_as_float(0x7fffffff);
        }
      };
      if (diag) {
        // Software-pipelined: the cost of step t - 1 is formed beside step
        // t's candidate control (one straight block, so the two chains
        // overlap); its rare non-finite fix-up and the sums follow the
        // dynamics step. The sums take the same terms in the same order.
        float pt[NT];  // tau of step t - 1 (zero before the first step; its cost is not added)
#pragma unroll
        for (int k = 0; k < NT; ++k) pt[k] = 0.0f;
        for (int t = 0; t < T; ++t) {
          float lp, qp;
          diag_cost(pt, t > 0 ? t - 1 : 0, lp, qp);
          float xb[NX], ub[NU], kt[NU], u[NU];
          load_rec(reinterpret_cast<const float4*>(REC + PREC_F * t), xb, ub);
          const float4* ks = reinterpret_cast<const float4*>(KS + PKS_F * t);
          {
            const float4 k4 = ks[NX];
            kt[0] = k4.x; kt[1] = k4.y; kt[2] = k4.z; kt[3] = k4.w;
          }
          candidate_u_reg(x, xb, ub, [&](int jj) { return ks[jj]; }, kt, al, bounds, blo, bhi, u);
          if (keep) store_rec(W.rec(cs, t), x, u);
          float tau[NT];
#pragma unroll
          for (int k = 0; k < NX; ++k) tau[k] = x[k] - xref(t, k);
#pragma unroll
          for (int a = 0; a < NU; ++a) tau[NX + a] = u[a] - uref(t, a);
          float xn[NX];
          drone_step(x, u, dt, xn);
#pragma unroll
          for (int k = 0; k < NX; ++k) x[k] = xn[k];
          if (t > 0) {
            nan_fix(pt, qp);
            sq += qp;
            sl += lp;
          }
#pragma unroll
          for (int k = 0; k < NT; ++k) pt[k] = tau[k];
        }
        float lp, qp;
        diag_cost(pt, T - 1, lp, qp);
        nan_fix(pt, qp);
        sq += qp;
        sl += lp;
      } else {
        cpipe.issue(0);
        if (T >= 2) cpipe.issue(1);
        for (int t = 0; t < T; ++t) {
          if (t + 2 < T) {
            cpipe.issue(t + 2);
            cp_async_wait<2>();
          } else if (t + 1 < T) {
            cp_async_wait<1>();
          } else {
            cp_async_wait<0>();
          }
          __syncwarp();
          float xb[NX], ub[NU], kt[NU], u[NU];
          load_rec(reinterpret_cast<const float4*>(REC + PREC_F * t), xb, ub);
          const float4* ks = reinterpret_cast<const float4*>(KS + PKS_F * t);
          {
            const float4 k4 = ks[NX];
            kt[0] = k4.x; kt[1] = k4.y; kt[2] = k4.z; kt[3] = k4.w;
          }
          candidate_u_reg(x, xb, ub, [&](int jj) { return ks[jj]; }, kt, al, bounds, blo, bhi, u);
          if (keep) store_rec(W.rec(cs, t), x, u);
          float tau[NT];
#pragma unroll
          for (int k = 0; k < NX; ++k) tau[k] = x[k] - xref(t, k);
#pragma unroll
          for (int a = 0; a < NU; ++a) tau[NX + a] = u[a] - uref(t, a);
          float l;
          {
            const float4* c4 = reinterpret_cast<const float4*>(CR + PCR_F * t + 16);
            const float4 h0 = c4[0], h1 = c4[1], h2 = c4[2], h3 = c4[3];
            const float cvv[NT] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z,
                                   h1.w, h2.x, h2.y, h2.z, h2.w, h3.x, h3.y};
            l = cvv[0] * tau[0];
#pragma unroll
            for (int jj = 1; jj < NT; ++jj) l = fmaf(cvv[jj], tau[jj], l);
          }
          float q = 0.0f;
          {
            const float* Ce = cpipe.block(t);
#pragma unroll
            for (int k = 0; k < NT; ++k) {
              const float2* r2 = reinterpret_cast<const float2*>(Ce + k * NT);
              float r = 0.0f;
#pragma unroll
              for (int jj = 0; jj < NT / 2; ++jj) {
                const float2 c2 = r2[jj];
                r = (jj == 0) ? c2.x * tau[0] : fmaf(c2.x, tau[2 * jj], r);
                r = fmaf(c2.y, tau[2 * jj + 1], r);
              }
              q = fmaf(tau[k], r, q);
            }
            __syncwarp();  // block t is read; the next issue may overwrite it
          }
          sq += q;
          sl += l;
          float xn[NX];
          drone_step(x, u, dt, xn);
#pragma unroll
          for (int k = 0; k < NX; ++k) x[k] = xn[k];
        }
      }
      if (keep) store_rec_x(W.rec(cs, T), x);
      float tn[NX];
#pragma unroll
      for (int k = 0; k < NX; ++k) tn[k] = x[k] - xref(T, k);
      const float mine = (0.5f * sq + sl) + terminal_cost(Cf, cf, tn);
#pragma unroll
      for (int jj = 0; jj < ILQR_MAX_ALPHAS_DEV; ++jj) {
        const float cj = __shfl_sync(FULL, mine, base + jj);
        if (jj >= p.n_alpha) continue;
        cand[jj] = cj;
        if (!nan_seen) {
          if (cj != cj) {
            nan_seen = true;
            jbest = jj;
            cmin = cj;
          } else if (!have || cj < cmin) {
            have = true;
            jbest = jj;
            cmin = cj;
          }
        }
      }
    }

    // ---- decision ---------------------------------------------------------------
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
      if (p.trace != nullptr && writer) p.trace[b * p.max_iter + it] = (int8_t)(accept ? jsel : -(jbest + 1));
      if (!accept && stall_iter == p.max_iter) {
        stall_iter = it;
        stall_gap = fabsf(cmin - best);
      }
      if (accept) best = cand[jsel];
      if (!accept && p.forced == nullptr) active = false;
    }
    const bool rerun = accept && jsel >= SOLVE_SLOTS - 1;
    if (accept && !rerun) nom = jsel < nom ? jsel : jsel + 1;
    if (__any_sync(FULL, rerun)) {
      const int dst = nom == 0 ? 1 : 0;
      if (rerun && writer) {
        const float al = p.alphas[jsel];
        float x[NX];
        load_x0(x);
        for (int t = 0; t < T; ++t) {
          float xb[NX], ub[NU], kt[NU], u[NU];
          load_rec(reinterpret_cast<const float4*>(REC + PREC_F * t), xb, ub);
          const float4* ks = reinterpret_cast<const float4*>(KS + PKS_F * t);
          const float4 k4 = ks[NX];
          kt[0] = k4.x; kt[1] = k4.y; kt[2] = k4.z; kt[3] = k4.w;
          candidate_u_reg(x, xb, ub, [&](int jj) { return ks[jj]; }, kt, al, bounds, blo, bhi, u);
          store_rec(W.rec(dst, t), x, u);
          float xn[NX];
          drone_step(x, u, dt, xn);
#pragma unroll
          for (int k = 0; k < NX; ++k) x[k] = xn[k];
        }
        store_rec_x(W.rec(dst, T), x);
      }
      if (rerun) nom = dst;
      __syncwarp();
    }
  }

  // ---- outputs (the 16 lanes of the half split the writes) ------------------------
  bool finite = true;
  if (valid) {
    const float* nrec = reinterpret_cast<const float*>(W.rec(nom, 0));
    const int64_t rstride = p.S * TRJ_REC;
#pragma unroll 4
    for (int f = i; f < (T + 1) * NX; f += HALF) {
      const int t = f / NX, k = f - t * NX;
      const float xv = nrec[t * rstride + k];
      finite &= isfinite(xv);
      p.X[b * (T + 1) * NX + f] = xv;
    }
#pragma unroll 4
    for (int f = i; f < T * NU; f += HALF) {
      const int t = f / NU, a = f - t * NU;
      const float uv = nrec[t * rstride + NX + a];
      finite &= isfinite(uv);
      p.U[b * T * NU + f] = uv;
      if (p.tight != nullptr) {
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
  const unsigned bad = __ballot_sync(FULL, !finite);
  if ((bad >> base) & 0xffffu) status |= ELEM_NONFINITE;
  if (diag) status |= ELEM_DIAG_COST;
  if (writer) {
    if (p.iters) p.iters[b] = iters;
    if (p.status) p.status[b] = status;
    if (p.best_cost) p.best_cost[b] = best;
    if (p.stall_iter) p.stall_iter[b] = stall_iter;
    if (p.stall_gap) p.stall_gap[b] = stall_gap;
  }
}

}  // namespace

size_t solve_smem_bytes(int tier) {
  const size_t base = (size_t)EPW * CBLK * 4 + (size_t)EPW * XS * 4;
  if (tier == TIER_MID) return base + STG_OFF + 2 * EPW * STG_F * 4;
  if (tier == TIER_LO) return base + STG_OFF + 2 * EPW * 40 * 4;
  return base + sizeof(uint64_t);
}

size_t solve_pair_smem_bytes(int T) {
  return (size_t)EPWP * pair_area(T, PREC_F + PJT_F + PKS_F + PCR_F, CBLK) * sizeof(float);
}


cudaError_t launch_solve(const CUtensorMap& tmC, const SolveParams& p, cudaStream_t stream) {
  const bool ref = p.x_ref != nullptr || p.u_ref != nullptr;
  if (p.T <= PAIR_MAX_T && (p.layout == LAYOUT_PAIR || (p.layout == LAYOUT_AUTO && p.B <= PAIR_MAX_B))) {
    const unsigned pgrid = (unsigned)((p.B + EPWP - 1) / EPWP);
    const size_t psmem = solve_pair_smem_bytes(p.T);
    cudaError_t e = ref ? allow_smem<solve_pair_kernel<true, 8>>(psmem) : allow_smem<solve_pair_kernel<false, 8>>(psmem);
    if (e != cudaSuccess) return e;
    if (ref) solve_pair_kernel<true, 8><<<pgrid, WARP, psmem, stream>>>(p);
    else solve_pair_kernel<false, 8><<<pgrid, WARP, psmem, stream>>>(p);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((p.B + EPW - 1) / EPW);
  auto launch = [&](const SolveParams& q, int tier) {
    const size_t smem = solve_smem_bytes(tier);
    if (ref) {
      if (tier == TIER_HI) solve_kernel<TEAM, true, TIER_HI><<<grid, WARP, smem, stream>>>(tmC, q);
      else if (tier == TIER_MID) solve_kernel<TEAM, true, TIER_MID><<<grid, WARP, smem, stream>>>(tmC, q);
      else solve_kernel<TEAM, true, TIER_LO><<<grid, WARP, smem, stream>>>(tmC, q);
    } else {
      if (tier == TIER_HI) solve_kernel<TEAM, false, TIER_HI><<<grid, WARP, smem, stream>>>(tmC, q);
      else if (tier == TIER_MID) solve_kernel<TEAM, false, TIER_MID><<<grid, WARP, smem, stream>>>(tmC, q);
      else solve_kernel<TEAM, false, TIER_LO><<<grid, WARP, smem, stream>>>(tmC, q);
    }
    return cudaGetLastError();
  };
  // Batches beyond one 8-CTA wave run as a chain of launches, each later one
  // on the elements still improving, compacted six per warp, at 12 CTAs per
  // SM (each list is a fraction of the batch and its count is known only on
  // the device; CTAs beyond it return at once). Up to 5 iterations: one split,
  // after max_iter - 2 (B200, T = 20, 5 iterations: a split after 3 beat
  // splits after 2 or 4, and chains of three or more launches, at B = 8192,
  // 12288 and 16384). More iterations: a launch per iteration after the first
  // (B = 65536, T = 50, 8 iterations, mean 1.78 run: 6.38 ms against 9.34
  // with the first launch at 3 iterations and 11.6 with one split after 6;
  // B = 32768, T = 10, 10 iterations: 1.41 ms against 1.74).
  const bool segmented = p.segment != 0 && p.forced == nullptr && p.max_iter >= 4 && grid > (unsigned)(SMS * TIER_HI);
  if (!segmented) {
    SolveParams q = p;
    q.seg_in = q.seg_out = -1;
    return launch(q, pick_solve_tier(grid));
  }
  const bool one_split = p.max_iter <= 5;
  SolveParams q = p;
  int it0 = 0;
  for (int k = 0; it0 < p.max_iter; ++k) {
    const int it1 = k == 0 ? (one_split ? p.max_iter - 2 : 1) : (one_split ? p.max_iter : it0 + 1);
    q.seg_in = k == 0 ? -1 : (k - 1) % 2;
    q.seg_out = it1 < p.max_iter ? k % 2 : -1;
    q.seg_it0 = it0;
    q.seg_it1 = it1;
    if (q.seg_out >= 0) {
      const cudaError_t e = cudaMemsetAsync(seg_count(p.ws, p.T, p.S, q.seg_out), 0, sizeof(int), stream);
      if (e != cudaSuccess) return e;
    }
    const cudaError_t e = launch(q, k == 0 ? pick_solve_tier(grid) : TIER_MID);
    if (e != cudaSuccess) return e;
    it0 = it1;
  }
  return cudaSuccess;
}

}  // namespace ilqr
