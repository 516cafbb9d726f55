// ilqr_fastmpc_abi.cu -- extern "C" entry points of the FastMPC numerics mode
// (declared in include/ilqr_b200.h). Arguments are validated on the host
// before anything is enqueued.
#include <cstring>

#include "ilqr_b200.h"
#include "ilqr_kernels.h"

namespace {

bool aligned16_fm(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

void cost_strides(int64_t B, int32_t T, int32_t layout, int64_t& bs, int64_t& ts) {
  bs = layout == ILQR_COST_TIME_MAJOR ? 1 : (int64_t)T;
  ts = layout == ILQR_COST_TIME_MAJOR ? B : 1;
}

}  // namespace

extern "C" {

int ilqr_b200_fastmpc_solve_workspace_size(int64_t B, int32_t T, int32_t n_alpha, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON || n_alpha < 1 ||
      n_alpha > ILQR_MAX_ALPHAS)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = ilqr::fm::solve_ws_bytes(B, T, n_alpha);
  return ILQR_OK;
}

int ilqr_b200_fastmpc_backward_workspace_size(int64_t B, int32_t T, size_t* bytes) {
  if (bytes == nullptr || B < 0 || B > ILQR_MAX_BATCH || T < 1 || T > ILQR_MAX_HORIZON)
    return ILQR_ERR_INVALID_ARGUMENT;
  *bytes = ilqr::fm::backward_ws_bytes(B, T);
  return ILQR_OK;
}

int ilqr_b200_fastmpc_solve_f32(const float* x0, const float* U_init, const float* C, const float* c,
                                const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
                                const float* u_min, const float* u_max, int64_t B, int32_t T, float dt,
                                int32_t max_iter, float reg_eps, float converge_tol, const float* alphas,
                                int32_t n_alpha, int32_t cost_layout, const int8_t* forced_trace,
                                int32_t forced_stop, float* X, float* U, uint8_t* tight_mask, float* X_lin,
                                float* U_lin, int8_t* trace, float* best_cost, int32_t* batch_info,
                                void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (B < 0 || T < 1 || max_iter < 0 || n_alpha < 1 || n_alpha > ILQR_MAX_ALPHAS || alphas == nullptr)
    return ILQR_ERR_INVALID_ARGUMENT;
  if (cost_layout != ILQR_COST_BATCH_MAJOR && cost_layout != ILQR_COST_TIME_MAJOR) return ILQR_ERR_INVALID_ARGUMENT;
  if ((u_min == nullptr) != (u_max == nullptr)) return ILQR_ERR_INVALID_ARGUMENT;
  if (forced_stop < 0 || forced_stop > max_iter || (forced_stop > 0 && forced_trace == nullptr))
    return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!x0 || !U_init || !C || !c || !X || !U) return ILQR_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  if (const int q = ilqr_b200_fastmpc_solve_workspace_size(B, T, n_alpha, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  if (!aligned16_fm(workspace)) return ILQR_ERR_MISALIGNED;
  ilqr::fm::FmSolveParams p;
  std::memset(&p, 0, sizeof(p));
  p.x0 = x0; p.U_init = U_init; p.C = C; p.c = c; p.C_final = C_final; p.c_final = c_final;
  p.x_ref = x_ref; p.u_ref = u_ref; p.u_min = u_min; p.u_max = u_max;
  p.B = B; p.T = T; p.dt = dt; p.max_iter = max_iter; p.reg = reg_eps; p.tol = converge_tol;
  p.n_alpha = n_alpha;
  for (int i = 0; i < n_alpha; ++i) p.alphas[i] = alphas[i];
  cost_strides(B, T, cost_layout, p.cost_bstride, p.cost_tstride);
  p.forced = forced_trace; p.forced_stop = forced_stop;
  p.X = X; p.U = U; p.X_lin = X_lin; p.U_lin = U_lin; p.tight = tight_mask; p.trace = trace;
  p.best_cost = best_cost;
  ilqr::fm::carve_solve(p, workspace);
  cudaError_t e = ilqr::fm::launch_solve(p, stream);
  if (e == cudaSuccess && batch_info != nullptr)
    e = cudaMemcpyAsync(batch_info, p.flags + 1, 2 * sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
  return e == cudaSuccess ? ILQR_OK : ILQR_ERR_CUDA;
}

int ilqr_b200_fastmpc_backward_f32(const float* X, const float* U, const float* X_lin, const float* U_lin,
                                   const float* C, const float* C_final, const float* x_ref, const float* u_ref,
                                   const uint8_t* tight_mask, const float* grad_X, const float* grad_U, int64_t B,
                                   int32_t T, float dt, float reg_eps, int32_t cost_layout, float* grad_x0,
                                   float* grad_C, float* grad_c, float* grad_C_final, float* grad_c_final,
                                   float* grad_x_ref, float* grad_u_ref, void* workspace, size_t workspace_bytes,
                                   cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (cost_layout != ILQR_COST_BATCH_MAJOR && cost_layout != ILQR_COST_TIME_MAJOR) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!X || !U || !X_lin || !U_lin || !C || !grad_X || !grad_U) return ILQR_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  if (const int q = ilqr_b200_fastmpc_backward_workspace_size(B, T, &need); q != ILQR_OK) return q;
  if (workspace == nullptr || workspace_bytes < need) return ILQR_ERR_WORKSPACE;
  if (!aligned16_fm(workspace)) return ILQR_ERR_MISALIGNED;
  ilqr::fm::FmBackwardParams p;
  std::memset(&p, 0, sizeof(p));
  p.X = X; p.U = U; p.X_lin = X_lin; p.U_lin = U_lin; p.C = C; p.C_final = C_final; p.x_ref = x_ref;
  p.u_ref = u_ref; p.tight = tight_mask; p.grad_X = grad_X; p.grad_U = grad_U;
  p.B = B; p.T = T; p.dt = dt; p.reg = reg_eps;
  cost_strides(B, T, cost_layout, p.cost_bstride, p.cost_tstride);
  p.grad_x0 = grad_x0; p.grad_C = grad_C; p.grad_c = grad_c; p.grad_C_final = grad_C_final;
  p.grad_c_final = grad_c_final; p.grad_x_ref = grad_x_ref; p.grad_u_ref = grad_u_ref;
  p.gains = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  const cudaError_t e = ilqr::fm::launch_backward(p, stream);
  return e == cudaSuccess ? ILQR_OK : ILQR_ERR_CUDA;
}

int ilqr_b200_fastmpc_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt, float* A,
                                    float* Bm, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!X || !U || !A || !Bm) return ILQR_ERR_INVALID_ARGUMENT;
  return ilqr::fm::launch_linearize(X, U, B, T, dt, A, Bm, stream) == cudaSuccess ? ILQR_OK : ILQR_ERR_CUDA;
}

int ilqr_b200_fastmpc_adjoint_lqr_f32(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                                      const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                                      const float* l_xN, const uint8_t* tight_mask, int64_t B, int32_t T,
                                      float reg_eps, float* K, float* k, float* v0, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!A || !Bm || !l_xx || !l_uu || !l_xu || !l_x || !l_u || !l_xxN || !l_xN || !K || !k || !v0)
    return ILQR_ERR_INVALID_ARGUMENT;
  return ilqr::fm::launch_adjoint_lqr(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN, tight_mask, B, T, reg_eps, K, k,
                                      v0, stream) == cudaSuccess
             ? ILQR_OK
             : ILQR_ERR_CUDA;
}

int ilqr_b200_fastmpc_assembly_f32(const float* K, const float* k, const float* v0, const float* A, const float* Bm,
                                   const float* X, const float* U, const float* x_ref, const float* u_ref, int64_t B,
                                   int32_t T, float* grad_C, float* grad_c, float* grad_x0, float* grad_x_ref,
                                   float* grad_u_ref, float* grad_C_final, float* grad_c_final, cudaStream_t stream) {
  if (B < 0 || T < 1) return ILQR_ERR_INVALID_ARGUMENT;
  if (B == 0) return ILQR_OK;
  if (!K || !k || !v0 || !A || !Bm || !X || !U || !grad_C || !grad_c || !grad_x0) return ILQR_ERR_INVALID_ARGUMENT;
  return ilqr::fm::launch_assembly(K, k, v0, A, Bm, X, U, x_ref, u_ref, B, T, grad_C, grad_c, grad_x0, grad_x_ref,
                                   grad_u_ref, grad_C_final, grad_c_final, stream) == cudaSuccess
             ? ILQR_OK
             : ILQR_ERR_CUDA;
}

}  // extern "C"
