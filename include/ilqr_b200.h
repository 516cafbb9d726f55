/*
 * ilqr_b200.h -- C ABI of the B200 batched differentiable iLQR solver for the
 * 10-state collective-thrust/body-rate quadrotor model.
 *
 * Every entry point takes plain device pointers to float32 arrays laid out
 * exactly as the reference's torch extension lays out its tensors (row-major,
 * batch first), sizes, and a cudaStream_t. Work is enqueued on that stream;
 * nothing is synchronised. Outputs are caller-owned. Scratch memory is a
 * caller-provided device workspace whose size the *_workspace_size query
 * reports. Functions return an ilqr_status_t and never throw.
 *
 * Numerics follow the reference's DiffMPC PyTorch implementation
 * (DifferentialMPC/controller.py) on the DroneDx CTBR model
 * (acmpc_public-master/diff_mpc_drones/drone.py:409-540).
 *
 * Each declaration names the reference interface it replaces.
 */
#ifndef ILQR_B200_H
#define ILQR_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ILQR_B200_ABI_VERSION 1
#define ILQR_NX 10
#define ILQR_NU 4
#define ILQR_N 14
#define ILQR_MAX_ALPHAS 8
#define ILQR_TRACE_NOT_RUN (-128)
/* Largest batch and horizon any entry point accepts. The workspace-size
 * queries reject larger ones with ILQR_ERR_INVALID_ARGUMENT before any size
 * arithmetic, so no byte count can wrap around. */
#define ILQR_MAX_BATCH ((int64_t)2147483647)
#define ILQR_MAX_HORIZON 65536

typedef enum {
  ILQR_OK = 0,
  ILQR_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, bad alphas */
  ILQR_ERR_MISALIGNED = 2,       /* C / grad_C not 16-byte aligned */
  ILQR_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  ILQR_ERR_CUDA = 4,             /* launch or driver-entry-point failure */
  ILQR_ERR_UNSUPPORTED_DEVICE = 5,
  ILQR_ERR_NOALLOC_LIMIT = 6     /* problem needs more than the fixed no-allocation scratch */
} ilqr_status_t;

/* Per-element status bits written to elem_status[b] by ilqr_b200_solve_f32. */
#define ILQR_ELEM_CHOL_FALLBACK 1u /* a Q_uu Cholesky failed; SVD inverse used */
#define ILQR_ELEM_NONFINITE 2u     /* X or U of the returned solution not finite */
#define ILQR_ELEM_PIPE_TIMEOUT 4u  /* an on-chip copy wait gave up (results invalid) */
#define ILQR_ELEM_DIAG_COST 8u     /* C blocks were diagonal: passes after the first read their diagonals only */

int ilqr_b200_abi_version(void);
const char* ilqr_b200_status_string(int status);

/* Returns ILQR_OK if `device` is a compute-capability 10.0 GPU. */
int ilqr_b200_check_device(int device);

/* Device workspace needed by ilqr_b200_solve_f32 for a batch B and horizon T. */
int ilqr_b200_solve_workspace_size(int64_t B, int32_t T, size_t* bytes);

/*
 * Full iLQR solve for a batch of B independent elements.
 * Replaces drone_ilqr_solve (differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:664-1064)
 * with the semantics of DifferentiableMPCController.solve_step
 * (DifferentialMPC/controller.py:303-435).
 *
 * Inputs (device, float32, row-major):
 *   x0 [B,10], U_init [B,T,4], C [B,T,14,14] (16-byte aligned), c [B,T,14],
 *   C_final [B,14,14] or NULL (zeros), c_final [B,14] or NULL (zeros),
 *   x_ref [B,T+1,10] or NULL (zeros), u_ref [B,T,4] or NULL (zeros),
 *   u_min [4], u_max [4] or both NULL (no control bounds),
 *   forced_trace [B,max_iter] int8 or NULL: replay recorded line-search
 *   decisions instead of deciding (j >= 0 accept candidate j; other negative
 *   values reject and continue; ILQR_TRACE_NOT_RUN stop).
 * alphas: HOST array of n_alpha (1..8) line-search step sizes.
 * Outputs (device): X [B,T+1,10], U [B,T,4], tight_mask [B,T,4] uint8
 *   (U within isclose(atol 1e-7, rtol 1e-5) of a bound).
 * Optional outputs (device, NULL to skip): trace [B,max_iter] int8,
 *   iters [B] int32 (iterations run), elem_status [B] uint32,
 *   best_cost [B] float, stall_iter [B] int32 (first rejected iteration or
 *   max_iter), stall_gap [B] float (|cost - best| at that rejection).
 * When every C_t block of a group of six consecutive elements is diagonal
 * (checked during the first pass), later passes read a compact copy of the
 * diagonals from the workspace instead of C; results are identical to the
 * dense path. The environment variable ILQR_B200_DIAG_CACHE=0 turns this off.
 */
int ilqr_b200_solve_f32(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * ilqr_b200_solve_f32 for callers that cannot allocate device memory. This
 * entry point has no counterpart in the reference: it exists for hosts that
 * must not allocate GPU memory while running (a control loop whose memory
 * budget is fixed at start-up, a plugin whose host owns the device
 * allocator). Same arguments and results as ilqr_b200_solve_f32 minus the
 * workspace: the scratch is a fixed ILQR_NOALLOC_SCRATCH_BYTES array inside
 * this library that every GPU loading the library holds until exit. Problems
 * whose ilqr_b200_solve_workspace_size exceeds it are rejected with
 * ILQR_ERR_NOALLOC_LIMIT (at T = 20 that is B > 1184). The entry point
 * allocates nothing. Its first call on a device looks up the array's device
 * address, so make that first call before any stream capture. All calls
 * share the array: calls that overlap on the GPU (other streams, other host
 * threads) race on it and must be serialised by the caller.
 */
#define ILQR_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int ilqr_b200_solve_f32_noalloc(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap, cudaStream_t stream);

/* Device workspace needed by ilqr_b200_backward_f32. */
int ilqr_b200_backward_workspace_size(int64_t B, int32_t T, size_t* bytes);

/*
 * n independent 4-dimensional box-constrained QPs,
 *   min 1/2 x^T H x + q^T x  s.t.  lower <= x <= upper,
 * by projected Newton, one thread per problem: mpc.pytorch's pnqp
 * (acmpc_public-master/mpc.pytorch/mpc/pnqp.py:5-84) with the reference
 * extension's per-problem settings (at most 10 Newton steps and 10 Armijo
 * trials, gamma 0.1, decay 0.1, ridge 1e-11, step tolerance 1e-4, bounds
 * active within 1e-8). Replaces drone_pnqp4_batch
 * (differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:1285-1316).
 * Inputs (device, float32): H [n,4,4], q, lower, upper [n,4], x_init [n,4] or
 * NULL (a zero row starts from the unconstrained solution).
 * Outputs: x_out [n,4], free_mask [n,4] (1 free, 0 held at a bound).
 */
int ilqr_b200_pnqp4_batch_f32(
    const float* H, const float* q, const float* lower, const float* upper,
    const float* x_init, int64_t n, float* x_out, float* free_mask, cudaStream_t stream);

/*
 * Fused implicit-differentiation backward at a solved (X, U): masked adjoint
 * Riccati, dX/dU sweep and gradient assembly in one kernel, with A_t, B_t
 * recomputed from (X_t, U_t) instead of read from memory.
 * Replaces DroneMPCFunction.backward (differentialMPCPerformance/mpc_compat.py:187-450)
 * plus drone_backward_pass_batched and drone_implicit_diff_assembly
 * (cpp/drone_ilqr_ext.cpp:1066-1177, 1221-1278), with the semantics of
 * ILQRSolve.backward / _zero_constrained_lqr (DifferentialMPC/controller.py:68-133,1006-1131).
 *
 * Inputs: X [B,T+1,10], U [B,T,4], C [B,T,14,14] (16-byte aligned),
 *   C_final [B,14,14] or NULL, x_ref [B,T+1,10] or NULL, u_ref [B,T,4] or NULL,
 *   tight_mask [B,T,4] uint8 or NULL (none tight), grad_X [B,T+1,10], grad_U [B,T,4].
 * Outputs (each NULL to skip): grad_x0 [B,10], grad_C [B,T,14,14] (16-byte
 *   aligned), grad_c [B,T,14], grad_C_final [B,14,14], grad_c_final [B,14],
 *   grad_x_ref [B,T+1,10] (row T is 0), grad_u_ref [B,T,4].
 */
int ilqr_b200_backward_f32(
    const float* X, const float* U, const float* C, const float* C_final,
    const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
    const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps,
    float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
    float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * ilqr_b200_solve_f32 / ilqr_b200_backward_f32 with time-major costs: C and
 * grad_C [T,B,14,14], c and grad_c [T,B,14] -- the layout of mpc.pytorch's
 * QuadCost, which the MPC operator receives (differentialMPCPerformance/
 * mpc_compat.py:80-96 copies it to batch-major). Every other argument, and
 * every result, as there; results equal those entry points' on the same costs.
 */
int ilqr_b200_solve_tm_f32(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

int ilqr_b200_backward_tm_f32(
    const float* X, const float* U, const float* C, const float* C_final,
    const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
    const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps,
    float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
    float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Costs from policy parameters. The policy builds its dense costs from a
 * sigmoid output s [B, 28 T] in a Python loop over t
 * (_build_cost_tensors, acmpc_public-master/training_modules/mlp_mpc_policy_diffmpc.py:194-247)
 * and then calls the solver; these two entry points replace that construction
 * plus ilqr_b200_solve_f32 / ilqr_b200_backward_f32 with the costs built
 * inside the kernels (28 instead of 210 floats per element and step read,
 * and a [B, 28 T] gradient written instead of grad_C).
 *
 * x_q = s[:, :14T] * range_q + cost_eps, x_p = s[:, 14T:]. x_q holds blocks of
 * T steps p (3), q (4), v (3), w (3), thrust (1); diag(C_t) is, in tau order
 * (p, q, v, thrust, w), the step-t slice of those blocks; c_t is
 * (x_p - 0.5) * range_p on the same slices except the thrust entry,
 * -(x_p * range_pt + cost_eps). The policy's values: cost_eps 0.1,
 * range_q = range_p = 1e5, range_pt = range_q * mass * 9.806. C_final, c_final,
 * x_ref, u_ref are zero (as in the policy). Everything else as
 * ilqr_b200_solve_f32 (same workspace size); results equal that entry point's
 * on the dense C, c the policy would build.
 */
int ilqr_b200_solve_sigmoid_f32(
    const float* x0, const float* U_init, const float* sigmoid_cost,
    float cost_eps, float range_q, float range_p, float range_pt,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Backward of ilqr_b200_solve_sigmoid_f32: as ilqr_b200_backward_f32, with
 * the gradient of the sigmoid cost row, grad_sigmoid_cost [B, 28 T] (NULL to
 * skip), in place of grad_C / grad_c: the chain rule of the construction
 * above applied to the diagonal of grad_C and to grad_c.
 */
int ilqr_b200_backward_sigmoid_f32(
    const float* X, const float* U, const float* sigmoid_cost,
    float cost_eps, float range_q, float range_p, float range_pt,
    const uint8_t* tight_mask, const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps,
    float* grad_x0, float* grad_sigmoid_cost,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * One step of the quadrotor model, x_next = f(x, u), for n states.
 * Replaces DroneDx.forward_CTBR (acmpc_public-master/diff_mpc_drones/drone.py:409-465)
 * and the reference's device step (cpp/forward_pass_kernel.cu:66-115).
 */
int ilqr_b200_dynamics_f32(const float* x, const float* u, int64_t n, float dt,
                           float* x_next, cudaStream_t stream);

/*
 * Discrete Jacobians A = I + dt J_x [B,T,10,10] and B = dt J_u [B,T,10,4] at
 * (X_t, U_t), t < T. Replaces drone_step_jacobian_kernel
 * (cpp/drone_kernels.cu:64-189) / DroneDx.grad_input (drone.py:524-540); used
 * to return A_lin, B_lin from the drone_ilqr_solve surface.
 */
int ilqr_b200_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt,
                            float* A, float* Bm, cudaStream_t stream);

/*
 * Masked adjoint Riccati for caller-supplied A [B,T,10,10], Bm [B,T,10,4],
 * l_xx [B,T,10,10], l_uu [B,T,4,4], l_xu [B,T,10,4], l_x [B,T,10],
 * l_u [B,T,4], l_xxN [B,10,10], l_xN [B,10], tight_mask [B,T,4] uint8 or NULL.
 * Outputs K [B,T,4,10], k [B,T,4], v0 [B,10].
 * Replaces drone_backward_pass_batched (cpp/drone_ilqr_ext.cpp:1066-1177),
 * with _zero_constrained_lqr semantics (controller.py:1035-1110).
 */
int ilqr_b200_adjoint_lqr_f32(
    const float* A, const float* Bm, const float* l_xx, const float* l_uu,
    const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
    const float* l_xN, const uint8_t* tight_mask, int64_t B, int32_t T, float reg_eps,
    float* K, float* k, float* v0, cudaStream_t stream);

/*
 * dX/dU sweep and gradient assembly from (K, k, v0) and A, Bm, X, U.
 * Replaces drone_implicit_diff_assembly (cpp/drone_ilqr_ext.cpp:1221-1278)
 * with ILQRSolve.backward semantics (controller.py:84-125). x_ref / u_ref may
 * be NULL (zeros). Outputs as for ilqr_b200_backward_f32 (each NULL to skip).
 */
int ilqr_b200_implicit_diff_assembly_f32(
    const float* K, const float* k, const float* v0, const float* A, const float* Bm,
    const float* X, const float* U, const float* x_ref, const float* u_ref,
    int64_t B, int32_t T,
    float* grad_C, float* grad_c, float* grad_x0, float* grad_x_ref,
    float* grad_u_ref, float* grad_C_final, float* grad_c_final, cudaStream_t stream);

/*
 * ---------------------------------------------------------------------------
 * 13-state rotor-thrust quadrotor. The reference's extension hard-codes the
 * 10-state CTBR model (cpp/drone_ilqr_ext.cpp:687-688); its DiffMPC solver
 * takes any model as f_dyn and linearises it by autodiff
 * (DifferentialMPC/controller.py:147-160, 607-615). These entry points are
 * that solver (same semantics as the 10-state entry points above) on the
 * rigid body x = [p (3), q (4, wxyz), v (3), w (3)] with four rotor thrusts
 * u in [0, 1] x 8.5 N, mass 0.75 kg, arm 0.15 m (X layout), inertia
 * diag(2.5e-3, 2.5e-3, 4.5e-3), explicit Euler step. tau = [x; u] has 17
 * entries: C [B,T,17,17], c [B,T,17], C_final [B,17,17], c_final [B,17],
 * x_ref [B,T+1,13], u_ref [B,T,4], X [B,T+1,13], U [B,T,4].
 * ---------------------------------------------------------------------------
 */

/* Device workspace of ilqr_b200_rotor13_solve_f32 (depends on n_alpha). */
int ilqr_b200_rotor13_solve_workspace_size(int64_t B, int32_t T, int32_t n_alpha, size_t* bytes);

/*
 * Batched solve on the rotor model: arguments, results and the per-element
 * decision outputs as ilqr_b200_solve_f32 (DiffMPC solve_step,
 * controller.py:303-435), with 13-state shapes. The workspace must be
 * 16-byte aligned. C needs no alignment.
 */
int ilqr_b200_rotor13_solve_f32(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Device workspace of ilqr_b200_rotor13_backward_f32. */
int ilqr_b200_rotor13_backward_workspace_size(int64_t B, int32_t T, size_t* bytes);

/*
 * Implicit-diff backward on the rotor model at a solved (X, U): as
 * ilqr_b200_backward_f32 (ILQRSolve.backward / _zero_constrained_lqr,
 * controller.py:68-133, 1006-1131) with 13-state shapes; every output may be
 * NULL. u_ref is accepted for symmetry and not read.
 */
int ilqr_b200_rotor13_backward_f32(
    const float* X, const float* U, const float* C, const float* C_final,
    const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
    const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps,
    float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
    float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* The rotor-model solve and backward with time-major costs (C, grad_C
 * [T,B,17,17], c, grad_c [T,B,17]); otherwise as the two entry points above. */
int ilqr_b200_rotor13_solve_tm_f32(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, const int8_t* forced_trace,
    float* X, float* U, uint8_t* tight_mask,
    int8_t* trace, int32_t* iters, uint32_t* elem_status, float* best_cost,
    int32_t* stall_iter, float* stall_gap,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

int ilqr_b200_rotor13_backward_tm_f32(
    const float* X, const float* U, const float* C, const float* C_final,
    const float* x_ref, const float* u_ref, const uint8_t* tight_mask,
    const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps,
    float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
    float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* One rotor-model step x_next = x + dt f(x, u) for n states [n,13], [n,4]. */
int ilqr_b200_rotor13_dynamics_f32(const float* x, const float* u, int64_t n, float dt,
                                   float* x_next, cudaStream_t stream);

/* Rotor-model Jacobians A [B,T,13,13], B [B,T,13,4] at (X_t, U_t), t < T. */
int ilqr_b200_rotor13_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt,
                                    float* A, float* Bm, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * FastMPC numerics mode: the solver as the reference FastMPC extension's CUDA
 * build runs it (differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:664-1064),
 * for the 10-state model. Differences from the DiffMPC entry points above:
 * the model step renormalises the quaternion; Q_uu carries the regulariser
 * once and gains come from a pivoted LU; with a control box every Riccati
 * step solves its box QP by PNQP-4 and masks the clamped controls
 * (backward_pass_kernel.cu:787-1047); the line search tries the given step
 * sizes (the reference's are 1, 0.5, 0.25, 0.1) with u = U + alpha k + K dx;
 * the batch stops as one when, at every fourth iteration or the last, the
 * largest cost improvement is below converge_tol.
 * ------------------------------------------------------------------------ */
#define ILQR_COST_BATCH_MAJOR 0 /* C [B,T,14,14], c [B,T,14] */
#define ILQR_COST_TIME_MAJOR 1  /* C [T,B,14,14], c [T,B,14] (QuadCost's layout) */

/* Device workspace of ilqr_b200_fastmpc_solve_f32. */
int ilqr_b200_fastmpc_solve_workspace_size(int64_t B, int32_t T, int32_t n_alpha, size_t* bytes);

/*
 * Replaces ext.drone_ilqr_solve of the reference's CUDA build
 * (drone_ilqr_ext.cpp:664-681 arguments, :1063 results). Inputs as
 * ilqr_b200_solve_f32 plus cost_layout (ILQR_COST_*). Outputs: X [B,T+1,10],
 * U [B,T,4], tight_mask [B,T,4] (the free mask of the last Riccati pass run,
 * inverted; zeros without a box), X_lin [B,T+1,10], U_lin [B,T,4] (where that
 * pass linearised: the point of the reference's returned A_lin, B_lin; the
 * backward needs them), trace [B,max_iter] (as ilqr_b200_solve_f32),
 * best_cost [B], batch_info [2] int32 on the device (converged flag,
 * iterations run). All outputs but X and U may be NULL. forced_trace with
 * forced_stop > 0 replays decisions and the batch's stop iteration.
 */
int ilqr_b200_fastmpc_solve_f32(
    const float* x0, const float* U_init, const float* C, const float* c,
    const float* C_final, const float* c_final, const float* x_ref, const float* u_ref,
    const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol,
    const float* alphas, int32_t n_alpha, int32_t cost_layout,
    const int8_t* forced_trace, int32_t forced_stop,
    float* X, float* U, uint8_t* tight_mask, float* X_lin, float* U_lin,
    int8_t* trace, float* best_cost, int32_t* batch_info,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Device workspace of ilqr_b200_fastmpc_backward_f32. */
int ilqr_b200_fastmpc_backward_workspace_size(int64_t B, int32_t T, size_t* bytes);

/*
 * Replaces the reference FastMPC operator's backward on its CUDA path
 * (differentialMPCPerformance/mpc_compat.py:188-258):
 * ext.drone_backward_pass_batched (drone_ilqr_ext.cpp:1066-1177, masked adjoint
 * Riccati at A, B of (X_lin, U_lin), l_x = -grad_X, l_u = -grad_U) then
 * ext.drone_implicit_diff_assembly (:1221-1278): grad_x0 = -v_0,
 * grad_C = -1/2 (d tau tau^T + tau d tau^T) with tau = [X - x_ref; U - u_ref],
 * grad_c = -d tau, grad_x_ref = dX (including t = T), grad_u_ref = dU,
 * grad_C_final, grad_c_final from the terminal tangent. Every output may be
 * NULL; grad_C and grad_c use cost_layout.
 */
int ilqr_b200_fastmpc_backward_f32(
    const float* X, const float* U, const float* X_lin, const float* U_lin,
    const float* C, const float* C_final, const float* x_ref, const float* u_ref,
    const uint8_t* tight_mask, const float* grad_X, const float* grad_U,
    int64_t B, int32_t T, float dt, float reg_eps, int32_t cost_layout,
    float* grad_x0, float* grad_C, float* grad_c, float* grad_C_final,
    float* grad_c_final, float* grad_x_ref, float* grad_u_ref,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * The reference FastMPC extension's separate entry points with its numerics
 * (the compatibility surface behind load_drone_ilqr_ext(numerics="fastmpc")).
 *
 * A [B,T,10,10], B [B,T,10,4] at (X_t, U_t), t < T: the Jacobian the
 * extension's drone_ilqr_solve returns as A_lin, B_lin
 * (drone_kernels.cu:64-190, drone_ilqr_ext.cpp:771-795).
 */
int ilqr_b200_fastmpc_linearize_f32(const float* X, const float* U, int64_t B, int32_t T, float dt,
                                    float* A, float* Bm, cudaStream_t stream);

/*
 * Replaces ext.drone_backward_pass_batched of the CUDA build
 * (drone_ilqr_ext.cpp:1066-1123, backward_pass_kernel.cu:617-745): masked
 * adjoint Riccati on caller-supplied matrices, reg once on Q_uu, a tight
 * control's row and column zeroed with a 1e-11 diagonal, pivoted-LU gains,
 * V = Q_xx + Q_xu K. tight_mask may be NULL. Outputs K [B,T,4,10], k [B,T,4],
 * v0 [B,10].
 */
int ilqr_b200_fastmpc_adjoint_lqr_f32(
    const float* A, const float* Bm, const float* l_xx, const float* l_uu, const float* l_xu,
    const float* l_x, const float* l_u, const float* l_xxN, const float* l_xN,
    const uint8_t* tight_mask, int64_t B, int32_t T, float reg_eps,
    float* K, float* k, float* v0, cudaStream_t stream);

/*
 * Replaces ext.drone_implicit_diff_assembly (drone_ilqr_ext.cpp:1221-1278,
 * backward_pass_kernel.cu:1092-1256): grad_x_ref includes t = T. x_ref, u_ref
 * and grad_x_ref, grad_u_ref, grad_C_final, grad_c_final may be NULL.
 */
int ilqr_b200_fastmpc_assembly_f32(
    const float* K, const float* k, const float* v0, const float* A, const float* Bm,
    const float* X, const float* U, const float* x_ref, const float* u_ref,
    int64_t B, int32_t T, float* grad_C, float* grad_c, float* grad_x0, float* grad_x_ref,
    float* grad_u_ref, float* grad_C_final, float* grad_c_final, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ILQR_B200_H */
