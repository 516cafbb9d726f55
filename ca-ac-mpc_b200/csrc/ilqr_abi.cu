// ilqr_abi.cu -- extern "C" entry points declared in include/ilqr_b200.h.
//
// Validation happens here, on the host, before anything is enqueued: every
// error is reported as a status code and nothing is launched on an invalid
// call. TMA descriptors for C (and grad_C) are encoded per call through the
// runtime's driver entry point, so the library does not link libcuda.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ilqr_b200.h"
#include "ilqr_kernels.h"
#include "ilqr_team.cuh"

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// View of a [B, T, 14, 14] (or, time-major, [T, B, 14, 14]) float tensor as
// {196, T, B}, box {196, 1, 6}: one box is the C_t blocks of the six elements
// a warp solves. The two layouts differ only in the strides of T and B.
int encode_cost_map(CUtensorMap* tm, const float* base, int64_t B, int32_t T, bool time_major) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ILQR_ERR_CUDA;
  const cuuint64_t dims[3] = {(cuuint64_t)ilqr::CBLK, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t blk = (cuuint64_t)ilqr::CBLK * 4u;
  const cuuint64_t strides[2] = {time_major ? (cuuint64_t)B * blk : blk, time_major ? blk : (cuuint64_t)T * blk};
  const cuuint32_t box[3] = {(cuuint32_t)ilqr::CBLK, 1u, (cuuint32_t)ilqr::EPW};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  std::memset(tm, 0, sizeof(*tm));
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ILQR_OK : ILQR_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? ILQR_OK : ILQR_ERR_CUDA; }

// ILQR_B200_LAYOUT=team|pair forces one kernel layout of the 10-state solve
// and backward (both give the same bits; the default picks by batch size).
int layout_from_env() {
  const char* v = std::getenv("ILQR_B200_LAYOUT");
  if (v == nullptr) return ilqr::LAYOUT_AUTO;
  if (std::strcmp(v, "team") == 0) return ilqr::LAYOUT_TEAM;
  if (std::strcmp(v, "pair") == 0) return ilqr::LAYOUT_PAIR;
  return ilqr::LAYOUT_AUTO;
}

}  // namespace

extern "C" {

int ilqr_b200_abi_version(void) { return ILQR_B200_ABI_VERSION; }

const char* ilqr_b200_status_string(int status) {
  switch (status) {
    case ILQR_OK: return "ok";
    case ILQR_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, size or step sizes)";
    case ILQR_ERR_MISALIGNED: return "C / grad_C must be 16-byte aligned";
    case ILQR_ERR_WORKSPACE: return "workspace missing or too small";
    case ILQR_ERR_CUDA: return "CUDA launch or driver entry point failure";
    case ILQR_ERR_UNSUPPORTED_DEVICE: return "device is not compute capability 10.0 (B200)";
    case ILQR_ERR_NOALLOC_LIMIT: return "problem too large for the fixed scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

int ilqr_b200_check_device(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return ILQR_ERR_CUDA;
  return (major == 10 && minor == 0) ? ILQR_OK : ILQR_ERR_UNSUPPORTED_DEVICE;
}

int ilqr_b200_solve_workspace_size(int64_t B, int32_t T, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)(ilqr::solve_ws_fields(T) * ilqr::ws_stride(B)) * sizeof(float);
  return ILQR_OK;
}

int ilqr_b200_backward_workspace_size(int64_t B, int32_t T, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)(ilqr::backward_ws_fields(T) * ilqr::ws_stride(B)) * sizeof(float);
  return ILQR_OK;
}

}  // extern "C"

namespace {

// Shared by the dense-cost and the sigmoid-cost solve: sig.p == nullptr means
// dense C, c (and optional terminal cost and references).
int solve_impl(const float* x0, const float* U_init, const float* C, const float* c, const float* C_final,
               const float* c_final, const float* x_ref, const float* u_ref, const ilqr::SigmoidCost& sig,
               const float* u_min, const float* u_max, int64_t B, int32_t T, float dt, int32_t max_iter,
               float reg_eps, const float* alphas, int32_t n_alpha, const int8_t* forced_trace, float* X, float* U,
               uint8_t* tight_mask, int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
               int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes, cudaStream_t stream,
               bool time_major = false) {
  if (B < 0 || T < 1 || max_iter < 0 || n_alpha < 1 || n_alpha > ILQR_MAX_ALPHAS || alphas == nullptr)
    return ILQR_ERR_INVALID_ARGUMENT;
  if ((u_min == nullptr) != (u_max == nullptr)) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!x0 || !U_init || !X || !U) return ILQR_ERR_INVALID_ARGUMENT;
  if (sig.p == nullptr) {
    if (!C || !c) return ILQR_ERR_INVALID_ARGUMENT;
    if (!aligned16(C)) return ILQR_ERR_MISALIGNED;
  }
  if ((C_final == nullptr) && (c_final != nullptr)) return ILQR_ERR_INVALID_ARGUMENT;
  // workspace records are indexed with 32-bit unsigned integers on the device
  {
    const int64_t recs = ilqr::SOLVE_SLOTS * ((int64_t)T + 1) > (int64_t)T * 10 ? ilqr::SOLVE_SLOTS * ((int64_t)T + 1)
                                                                                 : (int64_t)T * 10;
    if (recs * ilqr::ws_stride(B) >= ((int64_t)1 << 32)) return ILQR_ERR_INVALID_ARGUMENT;
  }
  size_t need = 0;
  if (const int q = ilqr_b200_solve_workspace_size(B, T, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  ilqr::SolveParams p{};
  p.x0 = x0; p.U_init = U_init; p.c = c; p.C_f = C_final; p.c_f = c_final;
  p.x_ref = x_ref; p.u_ref = u_ref; p.u_min = u_min; p.u_max = u_max; p.forced = forced_trace;
  p.X = X; p.U = U; p.tight = tight_mask; p.trace = trace; p.iters = iters; p.status = elem_status;
  p.best_cost = best_cost; p.stall_iter = stall_iter; p.stall_gap = stall_gap;
  p.ws = static_cast<float*>(workspace);
  p.B = B; p.S = ilqr::ws_stride(B); p.T = T; p.max_iter = max_iter; p.dt = dt; p.reg = reg_eps;
  for (int i = 0; i < n_alpha; ++i) p.alphas[i] = alphas[i];
  p.n_alpha = n_alpha;
  p.has_bounds = (u_min != nullptr) ? 1 : 0;
  const char* dc = std::getenv("ILQR_B200_DIAG_CACHE");
  p.diag_cache = (dc != nullptr && dc[0] == '0') ? 0 : 1;
  p.sig = sig;
  p.c_bstride = time_major ? ilqr::NT : (int64_t)T * ilqr::NT;
  p.c_tstride = time_major ? B * ilqr::NT : ilqr::NT;
  p.C = C;
  p.C_bstride = time_major ? 1 : (int64_t)T;
  p.C_tstride = time_major ? B : 1;
  p.layout = layout_from_env();
  // ILQR_B200_SEGMENT=0 keeps large team-layout solves in one launch (both
  // give the same bits)
  const char* sg = std::getenv("ILQR_B200_SEGMENT");
  p.segment = (sg != nullptr && sg[0] == '0') ? 0 : 1;
  p.seg_in = p.seg_out = -1;
  CUtensorMap tmC;
  std::memset(&tmC, 0, sizeof(tmC));  // never read in sigmoid mode (no pass copies C)
  if (sig.p == nullptr) {
    const int st = encode_cost_map(&tmC, C, B, T, time_major);
    if (st != ILQR_OK) return st;
  }
  return cuda_status(ilqr::launch_solve(tmC, p, stream));
}

int backward_impl(const float* X, const float* U, const float* C, const float* C_final, const float* x_ref,
                  const float* u_ref, const ilqr::SigmoidCost& sig, const uint8_t* tight_mask, const float* grad_X,
                  const float* grad_U, int64_t B, int32_t T, float dt, float reg_eps, float* grad_x0, float* grad_C,
                  float* grad_c, float* grad_C_final, float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
                  float* grad_sig, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                  bool time_major = false) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!X || !U || !grad_X || !grad_U) return ILQR_ERR_INVALID_ARGUMENT;
  if (sig.p == nullptr) {
    if (!C) return ILQR_ERR_INVALID_ARGUMENT;
    if (!aligned16(C) || (grad_C != nullptr && !aligned16(grad_C))) return ILQR_ERR_MISALIGNED;
  }
  size_t need = 0;
  if (const int q = ilqr_b200_backward_workspace_size(B, T, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  ilqr::BackwardParams p{};
  p.X = X; p.U = U; p.C_f = C_final; p.x_ref = x_ref; p.u_ref = u_ref; p.tight = tight_mask;
  p.gX = grad_X; p.gU = grad_U; p.g_x0 = grad_x0; p.g_c = grad_c; p.g_Cf = grad_C_final;
  p.g_cf = grad_c_final; p.g_xref = grad_x_ref; p.g_uref = grad_u_ref;
  p.ws = static_cast<float*>(workspace);
  p.B = B; p.S = ilqr::ws_stride(B); p.T = T; p.dt = dt; p.reg = reg_eps;
  p.write_gC = (sig.p == nullptr && grad_C != nullptr) ? 1 : 0;
  p.sig = sig;
  p.g_sig = grad_sig;
  p.gc_bstride = time_major ? ilqr::NT : (int64_t)T * ilqr::NT;
  p.gc_tstride = time_major ? B * ilqr::NT : ilqr::NT;
  p.C = C;
  p.g_C = p.write_gC ? grad_C : nullptr;
  p.C_bstride = time_major ? 1 : (int64_t)T;
  p.C_tstride = time_major ? B : 1;
  p.layout = layout_from_env();
  CUtensorMap tmC, tmG;
  std::memset(&tmC, 0, sizeof(tmC));  // never read in sigmoid mode
  std::memset(&tmG, 0, sizeof(tmG));
  if (sig.p == nullptr) {
    int st = encode_cost_map(&tmC, C, B, T, time_major);
    if (st != ILQR_OK) return st;
    st = encode_cost_map(&tmG, grad_C != nullptr ? grad_C : C, B, T, time_major);
    if (st != ILQR_OK) return st;
  }
  return cuda_status(ilqr::launch_backward(tmC, tmG, p, stream));
}

}  // namespace

extern "C" {

int ilqr_b200_solve_f32(const float* x0, const float* U_init, const float* C, const float* c,
                        const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
                        const float* u_min, const float* u_max, int64_t B, int32_t T, float dt, int32_t max_iter,
                        float reg_eps, float converge_tol, const float* alphas, int32_t n_alpha,
                        const int8_t* forced_trace, float* X, float* U, uint8_t* tight_mask, int8_t* trace,
                        int32_t* iters, uint32_t* elem_status, float* best_cost, int32_t* stall_iter,
                        float* stall_gap, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)converge_tol;  // global stopping only affects the reported flag; see stall_iter / stall_gap
  const ilqr::SigmoidCost none{nullptr, 0.0f, 0.0f, 0.0f, 0.0f};
  return solve_impl(x0, U_init, C, c, C_final, c_final, x_ref, u_ref, none, u_min, u_max, B, T, dt, max_iter,
                    reg_eps, alphas, n_alpha, forced_trace, X, U, tight_mask, trace, iters, elem_status, best_cost,
                    stall_iter, stall_gap, workspace, workspace_bytes, stream);
}

int ilqr_b200_solve_tm_f32(const float* x0, const float* U_init, const float* C, const float* c,
                           const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
                           const float* u_min, const float* u_max, int64_t B, int32_t T, float dt,
                           int32_t max_iter, float reg_eps, float converge_tol, const float* alphas,
                           int32_t n_alpha, const int8_t* forced_trace, float* X, float* U, uint8_t* tight_mask,
                           int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
                           int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  (void)converge_tol;
  const ilqr::SigmoidCost none{nullptr, 0.0f, 0.0f, 0.0f, 0.0f};
  return solve_impl(x0, U_init, C, c, C_final, c_final, x_ref, u_ref, none, u_min, u_max, B, T, dt, max_iter,
                    reg_eps, alphas, n_alpha, forced_trace, X, U, tight_mask, trace, iters, elem_status, best_cost,
                    stall_iter, stall_gap, workspace, workspace_bytes, stream, true);
}

int ilqr_b200_solve_sigmoid_f32(const float* x0, const float* U_init, const float* sigmoid_cost, float cost_eps,
                                float range_q, float range_p, float range_pt, const float* u_min,
                                const float* u_max, int64_t B, int32_t T, float dt, int32_t max_iter,
                                float reg_eps, float converge_tol, const float* alphas, int32_t n_alpha,
                                const int8_t* forced_trace, float* X, float* U, uint8_t* tight_mask,
                                int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
                                int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes,
                                cudaStream_t stream) {
  (void)converge_tol;
  if (B > 0 && sigmoid_cost == nullptr) return ILQR_ERR_INVALID_ARGUMENT;
  const ilqr::SigmoidCost sig{sigmoid_cost, cost_eps, range_q, range_p, range_pt};
  return solve_impl(x0, U_init, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, sig, u_min, u_max, B, T, dt,
                    max_iter, reg_eps, alphas, n_alpha, forced_trace, X, U, tight_mask, trace, iters, elem_status,
                    best_cost, stall_iter, stall_gap, workspace, workspace_bytes, stream);
}

int ilqr_b200_backward_f32(const float* X, const float* U, const float* C, const float* C_final,
                           const float* x_ref, const float* u_ref, const uint8_t* tight_mask, const float* grad_X,
                           const float* grad_U, int64_t B, int32_t T, float dt, float reg_eps, float* grad_x0,
                           float* grad_C, float* grad_c, float* grad_C_final, float* grad_c_final,
                           float* grad_x_ref, float* grad_u_ref, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  const ilqr::SigmoidCost none{nullptr, 0.0f, 0.0f, 0.0f, 0.0f};
  return backward_impl(X, U, C, C_final, x_ref, u_ref, none, tight_mask, grad_X, grad_U, B, T, dt, reg_eps, grad_x0,
                       grad_C, grad_c, grad_C_final, grad_c_final, grad_x_ref, grad_u_ref, nullptr, workspace,
                       workspace_bytes, stream);
}

int ilqr_b200_backward_tm_f32(const float* X, const float* U, const float* C, const float* C_final,
                              const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
                              const float* grad_X, const float* grad_U, int64_t B, int32_t T, float dt,
                              float reg_eps, float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
                              float* grad_c_final, float* grad_x_ref, float* grad_u_ref, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
  const ilqr::SigmoidCost none{nullptr, 0.0f, 0.0f, 0.0f, 0.0f};
  return backward_impl(X, U, C, C_final, x_ref, u_ref, none, tight_mask, grad_X, grad_U, B, T, dt, reg_eps, grad_x0,
                       grad_C, grad_c, grad_C_final, grad_c_final, grad_x_ref, grad_u_ref, nullptr, workspace,
                       workspace_bytes, stream, true);
}

int ilqr_b200_backward_sigmoid_f32(const float* X, const float* U, const float* sigmoid_cost, float cost_eps,
                                   float range_q, float range_p, float range_pt, const uint8_t* tight_mask,
                                   const float* grad_X, const float* grad_U, int64_t B, int32_t T, float dt,
                                   float reg_eps, float* grad_x0, float* grad_sigmoid_cost, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
  if (B > 0 && sigmoid_cost == nullptr) return ILQR_ERR_INVALID_ARGUMENT;
  const ilqr::SigmoidCost sig{sigmoid_cost, cost_eps, range_q, range_p, range_pt};
  return backward_impl(X, U, nullptr, nullptr, nullptr, nullptr, sig, tight_mask, grad_X, grad_U, B, T, dt,
                       reg_eps, grad_x0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, grad_sigmoid_cost,
                       workspace, workspace_bytes, stream);
}

int ilqr_b200_pnqp4_batch_f32(const float* H, const float* q, const float* lower, const float* upper,
                              const float* x_init, int64_t n, float* x_out, float* free_mask,
                              cudaStream_t stream) {
  if (n < 0) return ILQR_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!H || !q || !lower || !upper || !x_out || !free_mask)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status(ilqr::launch_pnqp4_batch(H, q, lower, upper, x_init, n, x_out, free_mask, stream));
}

int ilqr_b200_dynamics_f32(const float* x, const float* u, int64_t n, float dt, float* x_next,
                           cudaStream_t stream) {
  if (n < 0) return ILQR_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!x || !u || !x_next)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status(ilqr::launch_dynamics(x, u, n, dt, x_next, stream));
}

int ilqr_b200_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt, float* A, float* Bm,
                            cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B > 0 && (!X || !U || !A || !Bm)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status(ilqr::launch_linearize(X, U, B, T, dt, A, Bm, stream));
}

int ilqr_b200_adjoint_lqr_f32(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                              const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                              const float* l_xN, const uint8_t* tight_mask, int64_t B, int32_t T, float reg_eps,
                              float* K, float* k, float* v0, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B > 0 && (!A || !Bm || !l_xx || !l_uu || !l_xu || !l_x || !l_u || !l_xxN || !l_xN || !K || !k || !v0))
    return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status(ilqr::launch_adjoint_lqr(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN, tight_mask, B, T,
                                              reg_eps, K, k, v0, stream));
}

int ilqr_b200_implicit_diff_assembly_f32(const float* K, const float* k, const float* v0, const float* A,
                                         const float* Bm, const float* X, const float* U, const float* x_ref,
                                         const float* u_ref, int64_t B, int32_t T, float* grad_C, float* grad_c,
                                         float* grad_x0, float* grad_x_ref, float* grad_u_ref,
                                         float* grad_C_final, float* grad_c_final, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B > 0 && (!K || !k || !v0 || !A || !Bm || !X || !U)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status(ilqr::launch_assembly(K, k, v0, A, Bm, X, U, x_ref, u_ref, B, T, grad_C, grad_c, grad_x0,
                                           grad_x_ref, grad_u_ref, grad_C_final, grad_c_final, stream));
}

}  // extern "C"
