// ilqr_rotor13_abi.cu -- extern "C" entry points for the 13-state rotor-thrust
// model (declared in include/ilqr_b200.h). Validation on the host, before
// anything is enqueued, as for the 10-state entry points.
#include "ilqr_b200.h"
#include "ilqr_kernels.h"

namespace {

int cuda_status13(cudaError_t e) { return e == cudaSuccess ? ILQR_OK : ILQR_ERR_CUDA; }
bool aligned16_13(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace {

int r13_solve_impl(const float* x0, const float* U_init, const float* C, const float* c, const float* C_final,
                   const float* c_final, const float* x_ref, const float* u_ref, const float* u_min,
                   const float* u_max, int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps,
                   const float* alphas, int32_t n_alpha, const int8_t* forced_trace, float* X, float* U,
                   uint8_t* tight_mask, int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
                   int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream, bool time_major);
int r13_backward_impl(const float* X, const float* U, const float* C, const float* C_final, const float* x_ref,
                      const float* u_ref, const uint8_t* tight_mask, const float* grad_X, const float* grad_U,
                      int64_t B, int32_t T, float dt, float reg_eps, float* grad_x0, float* grad_C, float* grad_c,
                      float* grad_C_final, float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream, bool time_major);

}  // namespace

extern "C" {

int ilqr_b200_rotor13_solve_workspace_size(int64_t B, int32_t T, int32_t n_alpha, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON || n_alpha < 1 ||
      n_alpha > ILQR_MAX_ALPHAS)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)(ilqr::dense_solve_ws_fields(T, n_alpha) * B) * sizeof(float);
  return ILQR_OK;
}

int ilqr_b200_rotor13_backward_workspace_size(int64_t B, int32_t T, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)(ilqr::dense_backward_ws_fields(T) * B) * sizeof(float);
  return ILQR_OK;
}

int ilqr_b200_rotor13_solve_f32(const float* x0, const float* U_init, const float* C, const float* c,
                                const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
                                const float* u_min, const float* u_max, int64_t B, int32_t T, float dt,
                                int32_t max_iter, float reg_eps, float converge_tol, const float* alphas,
                                int32_t n_alpha, const int8_t* forced_trace, float* X, float* U, uint8_t* tight_mask,
                                int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
                                int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes,
                                cudaStream_t stream) {
  (void)converge_tol;  // the global flag is formed by the caller from stall_iter / stall_gap
  return r13_solve_impl(x0, U_init, C, c, C_final, c_final, x_ref, u_ref, u_min, u_max, B, T, dt, max_iter, reg_eps,
                        alphas, n_alpha, forced_trace, X, U, tight_mask, trace, iters, elem_status, best_cost,
                        stall_iter, stall_gap, workspace, workspace_bytes, stream, false);
}

int ilqr_b200_rotor13_solve_tm_f32(const float* x0, const float* U_init, const float* C, const float* c,
                                   const float* C_final, const float* c_final, const float* x_ref,
                                   const float* u_ref, const float* u_min, const float* u_max, int64_t B, int32_t T,
                                   float dt, int32_t max_iter, float reg_eps, float converge_tol,
                                   const float* alphas, int32_t n_alpha, const int8_t* forced_trace, float* X,
                                   float* U, uint8_t* tight_mask, int8_t* trace, int32_t* iters,
                                   uint32_t* elem_status, float* best_cost, int32_t* stall_iter, float* stall_gap,
                                   void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)converge_tol;
  return r13_solve_impl(x0, U_init, C, c, C_final, c_final, x_ref, u_ref, u_min, u_max, B, T, dt, max_iter, reg_eps,
                        alphas, n_alpha, forced_trace, X, U, tight_mask, trace, iters, elem_status, best_cost,
                        stall_iter, stall_gap, workspace, workspace_bytes, stream, true);
}

int ilqr_b200_rotor13_backward_f32(const float* X, const float* U, const float* C, const float* C_final,
                                   const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
                                   const float* grad_X, const float* grad_U, int64_t B, int32_t T, float dt,
                                   float reg_eps, float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
                                   float* grad_c_final, float* grad_x_ref, float* grad_u_ref, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
  return r13_backward_impl(X, U, C, C_final, x_ref, u_ref, tight_mask, grad_X, grad_U, B, T, dt, reg_eps, grad_x0,
                           grad_C, grad_c, grad_C_final, grad_c_final, grad_x_ref, grad_u_ref, workspace,
                           workspace_bytes, stream, false);
}

int ilqr_b200_rotor13_backward_tm_f32(const float* X, const float* U, const float* C, const float* C_final,
                                      const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
                                      const float* grad_X, const float* grad_U, int64_t B, int32_t T, float dt,
                                      float reg_eps, float* grad_x0, float* grad_C, float* grad_c,
                                      float* grad_C_final, float* grad_c_final, float* grad_x_ref,
                                      float* grad_u_ref, void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream) {
  return r13_backward_impl(X, U, C, C_final, x_ref, u_ref, tight_mask, grad_X, grad_U, B, T, dt, reg_eps, grad_x0,
                           grad_C, grad_c, grad_C_final, grad_c_final, grad_x_ref, grad_u_ref, workspace,
                           workspace_bytes, stream, true);
}

}  // extern "C"

namespace {

int r13_solve_impl(const float* x0, const float* U_init, const float* C, const float* c, const float* C_final,
                   const float* c_final, const float* x_ref, const float* u_ref, const float* u_min,
                   const float* u_max, int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps,
                   const float* alphas, int32_t n_alpha, const int8_t* forced_trace, float* X, float* U,
                   uint8_t* tight_mask, int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
                   int32_t* stall_iter, float* stall_gap, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream, bool time_major) {
  if (B < 0 || T < 1 || max_iter < 0 || n_alpha < 1 || n_alpha > ILQR_MAX_ALPHAS || alphas == nullptr)
    return ILQR_ERR_INVALID_ARGUMENT;
  if ((u_min == nullptr) != (u_max == nullptr)) return ILQR_ERR_INVALID_ARGUMENT;
  if ((C_final == nullptr) && (c_final != nullptr)) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!x0 || !U_init || !C || !c || !X || !U) return ILQR_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  if (const int q = ilqr_b200_rotor13_solve_workspace_size(B, T, n_alpha, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  if (!aligned16_13(workspace)) return ILQR_ERR_MISALIGNED;
  ilqr::DenseSolveParams p{};
  p.x0 = x0; p.U_init = U_init; p.C = C; p.c = c; p.C_f = C_final; p.c_f = c_final;
  p.x_ref = x_ref; p.u_ref = u_ref; p.u_min = u_min; p.u_max = u_max; p.forced = forced_trace;
  p.X = X; p.U = U; p.tight = tight_mask; p.trace = trace; p.iters = iters; p.status = elem_status;
  p.best_cost = best_cost; p.stall_iter = stall_iter; p.stall_gap = stall_gap;
  p.ws = static_cast<float*>(workspace);
  p.ws_fields = ilqr::dense_solve_ws_fields(T, n_alpha);
  p.B = B; p.T = T; p.max_iter = max_iter; p.dt = dt; p.reg = reg_eps;
  for (int i = 0; i < n_alpha; ++i) p.alphas[i] = alphas[i];
  p.n_alpha = n_alpha;
  p.has_bounds = (u_min != nullptr) ? 1 : 0;
  p.cost_bstride = time_major ? 1 : T;
  p.cost_tstride = time_major ? B : 1;
  return cuda_status13(ilqr::launch_dense_solve(p, stream));
}

int r13_backward_impl(const float* X, const float* U, const float* C, const float* C_final, const float* x_ref,
                      const float* u_ref, const uint8_t* tight_mask, const float* grad_X, const float* grad_U,
                      int64_t B, int32_t T, float dt, float reg_eps, float* grad_x0, float* grad_C, float* grad_c,
                      float* grad_C_final, float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream, bool time_major) {
  (void)u_ref;  // the backward does not depend on u_ref (the solution already does)
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!X || !U || !C || !grad_X || !grad_U) return ILQR_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  if (const int q = ilqr_b200_rotor13_backward_workspace_size(B, T, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  if (!aligned16_13(workspace)) return ILQR_ERR_MISALIGNED;
  ilqr::DenseBackwardParams p{};
  p.X = X; p.U = U; p.C = C; p.C_f = C_final; p.x_ref = x_ref; p.u_ref = u_ref; p.tight = tight_mask;
  p.gX = grad_X; p.gU = grad_U; p.g_x0 = grad_x0; p.g_C = grad_C; p.g_c = grad_c; p.g_Cf = grad_C_final;
  p.g_cf = grad_c_final; p.g_xref = grad_x_ref; p.g_uref = grad_u_ref;
  p.ws = static_cast<float*>(workspace);
  p.B = B; p.T = T; p.dt = dt; p.reg = reg_eps;
  p.cost_bstride = time_major ? 1 : T;
  p.cost_tstride = time_major ? B : 1;
  return cuda_status13(ilqr::launch_dense_backward(p, stream));
}

}  // namespace

extern "C" {

int ilqr_b200_rotor13_dynamics_f32(const float* x, const float* u, int64_t n, float dt, float* x_next,
                                   cudaStream_t stream) {
  if (n < 0) return ILQR_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!x || !u || !x_next)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status13(ilqr::launch_rotor13_dynamics(x, u, n, dt, x_next, stream));
}

int ilqr_b200_rotor13_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt, float* A,
                                    float* Bm, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B > 0 && (!X || !U || !A || !Bm)) return ILQR_ERR_INVALID_ARGUMENT;
  return cuda_status13(ilqr::launch_rotor13_linearize(X, U, B, T, dt, A, Bm, stream));
}

}  // extern "C"
