// TEST INFRASTRUCTURE ONLY -- extern "C" entry points over the reference
// FastMPC extension's CUDA kernels (differentialMPCPerformance/cpp:
// drone_kernels.cu, forward_pass_kernel.cu, backward_pass_kernel.cu,
// pnqp_kernel.cu), compiled from the reference's own sources with its own CUDA
// flags by oracle/build_fastmpc_ref.py into oracle/_ref/. Only the GPU parity
// tests load the result (through tests/fastmpc_ref.py), to check the B200
// FastMPC-numerics kernels against the reference's arithmetic. Nothing in the
// product links or calls this.
//
// The prototypes below restate the reference launchers' signatures
// (drone_kernels.cuh:11-31, forward_pass_kernel.cuh:57-73,
// backward_pass_kernel.cuh:102-230, the last defined in pnqp_kernel.cu:43); the wrappers only forward and report the
// launch status.
#include <cuda_runtime.h>

namespace drone_kernels {
void launch_drone_step_jacobian(const float* x, const float* u, float* x_next, float* A, float* B_mat, float dt,
                                int batch_size, cudaStream_t stream);
void launch_batched_rollout(const float* x0, const float* U, float* X, float dt, int batch_size, int horizon,
                            cudaStream_t stream);
void launch_forward_pass_fused(const float* x0, const float* X_nom, const float* U_nom, const float* K,
                               const float* k, const float* alphas, float dt, int batch_size, int num_alphas, int T,
                               bool has_bounds, const float* u_min, const float* u_max, float* X_out, float* U_out,
                               cudaStream_t stream);
void launch_backward_pass_batched(const float* A, const float* B, const float* l_xx, const float* l_uu,
                                  const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                                  const float* l_xN, const bool* tight_mask, float reg_eps, int batch_size, int T,
                                  float* K_out, float* k_out, float* v0_out, cudaStream_t stream);
void launch_backward_pass_batched_pnqp(const float* A, const float* B, const float* l_xx, const float* l_uu,
                                       const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                                       const float* l_xN, const float* U, const float* u_min, const float* u_max,
                                       float reg_eps, int batch_size, int T, float* K_out, float* k_out,
                                       float* v0_out, float* free_mask_out, cudaStream_t stream);
void launch_pnqp4_batch(const float* H, const float* q, const float* lower, const float* upper, const float* x_init,
                        float* x_out, float* free_mask_out, int N, cudaStream_t stream);
void launch_implicit_diff_assembly(const float* K_seq, const float* k_seq, const float* v0, const float* A_lin,
                                   const float* B_lin, const float* X, const float* U, const float* x_ref,
                                   const float* u_ref, float* grad_C, float* grad_c, float* grad_x0, float* grad_xref,
                                   float* grad_uref, float* grad_C_final, float* grad_c_final, int batch_size, int T,
                                   cudaStream_t stream);
}  // namespace drone_kernels

namespace {
int status() { return (int)cudaGetLastError(); }
cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

extern "C" {

int fmref_step_jacobian(const float* x, const float* u, float* x_next, float* A, float* Bm, float dt, int n,
                        void* s) {
  drone_kernels::launch_drone_step_jacobian(x, u, x_next, A, Bm, dt, n, st(s));
  return status();
}

int fmref_rollout(const float* x0, const float* U, float* X, float dt, int B, int T, void* s) {
  drone_kernels::launch_batched_rollout(x0, U, X, dt, B, T, st(s));
  return status();
}

int fmref_forward(const float* x0, const float* X, const float* U, const float* K, const float* k,
                  const float* alphas, float dt, int B, int n_alpha, int T, int has_bounds, const float* u_min,
                  const float* u_max, float* X_out, float* U_out, void* s) {
  drone_kernels::launch_forward_pass_fused(x0, X, U, K, k, alphas, dt, B, n_alpha, T, has_bounds != 0, u_min, u_max,
                                           X_out, U_out, st(s));
  return status();
}

int fmref_riccati(const float* A, const float* Bm, const float* lxx, const float* luu, const float* lxu,
                  const float* lx, const float* lu, const float* lxxN, const float* lxN, const unsigned char* tight,
                  float reg, int B, int T, float* K, float* k, float* v0, void* s) {
  drone_kernels::launch_backward_pass_batched(A, Bm, lxx, luu, lxu, lx, lu, lxxN, lxN,
                                              reinterpret_cast<const bool*>(tight), reg, B, T, K, k, v0, st(s));
  return status();
}

int fmref_riccati_pnqp(const float* A, const float* Bm, const float* lxx, const float* luu, const float* lxu,
                       const float* lx, const float* lu, const float* lxxN, const float* lxN, const float* U,
                       const float* u_min, const float* u_max, float reg, int B, int T, float* K, float* k,
                       float* v0, float* free_mask, void* s) {
  drone_kernels::launch_backward_pass_batched_pnqp(A, Bm, lxx, luu, lxu, lx, lu, lxxN, lxN, U, u_min, u_max, reg, B,
                                                   T, K, k, v0, free_mask, st(s));
  return status();
}

int fmref_pnqp4(const float* H, const float* q, const float* lo, const float* hi, const float* x_init, float* x,
                float* free_mask, int n, void* s) {
  drone_kernels::launch_pnqp4_batch(H, q, lo, hi, x_init, x, free_mask, n, st(s));
  return status();
}

int fmref_assembly(const float* K, const float* k, const float* v0, const float* A, const float* Bm, const float* X,
                   const float* U, const float* x_ref, const float* u_ref, float* gC, float* gc, float* gx0,
                   float* gxr, float* gur, float* gCf, float* gcf, int B, int T, void* s) {
  drone_kernels::launch_implicit_diff_assembly(K, k, v0, A, Bm, X, U, x_ref, u_ref, gC, gc, gx0, gxr, gur, gCf, gcf, B,
                                               T, st(s));
  return status();
}

}  // extern "C"
