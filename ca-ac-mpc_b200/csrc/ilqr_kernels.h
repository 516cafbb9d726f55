// ilqr_kernels.h -- host-side launch interface shared by the .cu files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define ILQR_MAX_ALPHAS_DEV 8

namespace ilqr {

// Diagonal quadratic costs given as the policy's sigmoid outputs [B, 28 T]
// (x_q = p[:, :14T], x_p = p[:, 14T:]): diag(C_t)_i = x_q * range_q + eps,
// c_t,i = (x_p - 0.5) range_p, and for the thrust entry -(x_p range_pt + eps).
struct SigmoidCost {
  const float* p;
  float eps, range_q, range_p, range_pt;
};

struct SolveParams {
  const float* x0;
  const float* U_init;
  const float* c;
  const float* C_f;
  const float* c_f;
  const float* x_ref;
  const float* u_ref;
  const float* u_min;
  const float* u_max;
  const int8_t* forced;
  float* X;
  float* U;
  uint8_t* tight;
  int8_t* trace;
  int32_t* iters;
  uint32_t* status;
  float* best_cost;
  int32_t* stall_iter;
  float* stall_gap;
  float* ws;
  int64_t B;
  int64_t S;  // workspace element stride (B rounded up to 32)
  int T;
  int max_iter;
  float dt;
  float reg;
  float alphas[ILQR_MAX_ALPHAS_DEV];
  int n_alpha;
  int has_bounds;
  int diag_cache;  // 1: detect diagonal C_t blocks and stop re-reading them after the first pass
  SigmoidCost sig;  // sig.p != nullptr: costs built from policy parameters (C, c unused)
  // floats between the c records of consecutive elements / steps: T * 14 / 14
  // for batch-major costs [B, T, 14], 14 / B * 14 for time-major [T, B, 14]
  int64_t c_bstride;
  int64_t c_tstride;
  // The pair layout (two elements per warp) copies C blocks with cp.async:
  // C itself and the blocks between consecutive elements / steps (T, 1)
  // batch-major, (1, B) time-major.
  const float* C;
  int64_t C_bstride;
  int64_t C_tstride;
  int layout;  // LAYOUT_AUTO, LAYOUT_TEAM or LAYOUT_PAIR
  int segment;  // 0: off; else large team-layout solves run as a chain of launches
  int seg_in;   // this launch resumes the elements of list seg_in (0, 1), or -1: all elements
  int seg_out;  // ... and defers those still improving at seg_it1 into list seg_out, or -1: none
  int seg_it0;  // iterations [seg_it0, seg_it1) of this launch
  int seg_it1;
};

// Segmented team solve. Elements stop after different numbers of iterations
// (B = 16384, T = 20, 5 iterations: 3.45 on average), while a warp of six runs
// until its last one stops (4.74 on average), so a third of the lanes idle.
// A chain of launches: the first runs every element for the first iterations;
// then, after each iteration, warps whose costs are diagonal stop, and each
// of their elements that is still improving saves its state (nominal slot,
// best cost, status bits) and enters a list that the next launch runs, six
// elements per warp. The arithmetic of every element is the same, so the
// results are the same bits. State, the two lists (alternating) and their
// counts live in floats 12..15 of the t = T records of slots 0, 1 and 3,
// and 2 and 4 (element 0's), which the solve never uses otherwise.

// Kernel layouts of the 10-state solve and backward. TEAM: six elements per
// warp, five lanes each (ilqr_team.cuh); PAIR: two elements per warp,
// sixteen lanes each (ilqr_pair.cuh). Both compute the same bits; AUTO picks
// PAIR for batches up to PAIR_MAX_B.
constexpr int LAYOUT_AUTO = 0, LAYOUT_TEAM = 1, LAYOUT_PAIR = 2;

struct BackwardParams {
  const float* X;
  const float* U;
  const float* C_f;
  const float* x_ref;
  const float* u_ref;
  const uint8_t* tight;
  const float* gX;
  const float* gU;
  float* g_x0;
  float* g_c;
  float* g_Cf;
  float* g_cf;
  float* g_xref;
  float* g_uref;
  float* ws;
  int64_t B;
  int64_t S;
  int T;
  float dt;
  float reg;
  int write_gC;
  SigmoidCost sig;  // sig.p != nullptr: costs from policy parameters; grad goes to g_sig
  float* g_sig;     // [B, 28 T] gradient of the parameters (sigmoid mode)
  int64_t gc_bstride;  // layout of grad_c, as SolveParams::c_bstride / c_tstride
  int64_t gc_tstride;
  const float* C;      // pair layout: C and grad_C blocks, strides as SolveParams::C_bstride
  float* g_C;
  int64_t C_bstride;
  int64_t C_tstride;
  int layout;
};

// Solve workspace, in floats, element-interleaved with stride S (the record
// of element b sits at (... * S + b) * width):
//   trajectory slots [SOLVE_SLOTS][T+1][S][16]: x[10], u[4], 2 pad (u unused at t = T)
//   gains K          [T][10][S][4]: column j of K_t (the 4 gains of state j)
//   feedforward k    [T][S][4]
//   cost records     [T][S][32]: the 14 diagonal entries of C_t, 2 pad, c_t (14), 2 pad
// One slot holds the nominal trajectory, the others the line-search candidates.
constexpr int SOLVE_SLOTS = 6;
constexpr int TRJ_REC = 16;
constexpr int COST_REC = 32;
inline int64_t solve_ws_fields(int T) {
  return (int64_t)SOLVE_SLOTS * (T + 1) * TRJ_REC + (int64_t)T * (10 * 4 + 4 + COST_REC);
}
// Backward workspace: K_t columns [T][10][S][4] and k_t [T][S][4].
inline int64_t backward_ws_fields(int T) { return (int64_t)T * (40 + 4); }
inline int64_t ws_stride(int64_t B) { return (B + 31) / 32 * 32; }

// The 13-state rotor-thrust model (ilqr_rotor13.cuh), solved by the dense
// row-per-lane kernels of ilqr_dense.cu. Dense inputs as the 10-state entry
// points, with 13 states and tau = [x; u] of length 17.
struct DenseSolveParams {
  const float* x0;
  const float* U_init;
  const float* C;
  const float* c;
  const float* C_f;
  const float* c_f;
  const float* x_ref;
  const float* u_ref;
  const float* u_min;
  const float* u_max;
  const int8_t* forced;
  float* X;
  float* U;
  uint8_t* tight;
  int8_t* trace;
  int32_t* iters;
  uint32_t* status;
  float* best_cost;
  int32_t* stall_iter;
  float* stall_gap;
  float* ws;
  int64_t ws_fields;  // floats of workspace per element
  int64_t B;
  int T;
  int max_iter;
  float dt;
  float reg;
  float alphas[ILQR_MAX_ALPHAS_DEV];
  int n_alpha;
  int has_bounds;
  // C blocks (and c records) between consecutive elements / steps: (T, 1)
  // batch-major [B, T, ...], (1, B) time-major [T, B, ...]
  int64_t cost_bstride;
  int64_t cost_tstride;
};

struct DenseBackwardParams {
  const float* X;
  const float* U;
  const float* C;
  const float* C_f;
  const float* x_ref;
  const float* u_ref;
  const uint8_t* tight;
  const float* gX;
  const float* gU;
  float* g_x0;
  float* g_C;
  float* g_c;
  float* g_Cf;
  float* g_cf;
  float* g_xref;
  float* g_uref;
  float* ws;
  int64_t B;
  int T;
  float dt;
  float reg;
  int64_t cost_bstride;  // C, c, grad_C, grad_c layout, as DenseSolveParams
  int64_t cost_tstride;
};

// Per-element workspace of the dense solve: (n_alpha + 1) trajectory slots of
// T + 1 records of 20 floats, then K_t columns and k_t as [T][14] float4.
int64_t dense_solve_ws_fields(int T, int n_alpha);
// Per-element workspace of the dense backward: K_t, k_t as [T][14] float4.
int64_t dense_backward_ws_fields(int T);
cudaError_t launch_dense_solve(const DenseSolveParams& p, cudaStream_t stream);
cudaError_t launch_dense_backward(const DenseBackwardParams& p, cudaStream_t stream);
cudaError_t launch_rotor13_dynamics(const float* x, const float* u, int64_t n, float dt, float* xn,
                                    cudaStream_t s);
cudaError_t launch_rotor13_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A,
                                     float* Bm, cudaStream_t s);

size_t solve_smem_bytes(int tier);
size_t backward_smem_bytes();
cudaError_t launch_solve(const CUtensorMap& tmC, const SolveParams& p, cudaStream_t stream);
cudaError_t launch_backward(const CUtensorMap& tmC, const CUtensorMap& tmG, const BackwardParams& p,
                            cudaStream_t stream);
cudaError_t launch_dynamics(const float* x, const float* u, int64_t n, float dt, float* xn, cudaStream_t s);
cudaError_t launch_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A, float* Bm,
                             cudaStream_t s);
cudaError_t launch_adjoint_lqr(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                               const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                               const float* l_xN, const uint8_t* tight, int64_t B, int T, float reg, float* K,
                               float* k, float* v0, cudaStream_t s);
cudaError_t launch_pnqp4_batch(const float* H, const float* q, const float* lower, const float* upper,
                               const float* x_init, int64_t n, float* x_out, float* free_mask, cudaStream_t stream);
cudaError_t launch_assembly(const float* K, const float* k, const float* v0, const float* A, const float* Bm,
                            const float* X, const float* U, const float* x_ref, const float* u_ref, int64_t B,
                            int T, float* gC, float* gc, float* gx0, float* gxr, float* gur, float* gCf,
                            float* gcf, cudaStream_t s);


// ---- FastMPC numerics mode (ilqr_fastmpc.cu) --------------------------------
namespace fm {

constexpr int FM_CHECK_PERIOD = 4;  // iterations between batch convergence checks

struct FmState {
  int32_t* nom;   // nominal slot
  int32_t* lin;   // slot of the last Riccati pass's linearisation point
  int32_t* code;  // 0 while improving, else the trace code of the freezing rejection
  float* best;    // best cost
  float* imp;     // |best before - best after| of the last iteration run
};

struct FmSolveParams {
  const float* x0;
  const float* U_init;
  const float* C;
  const float* c;
  const float* C_final;
  const float* c_final;
  const float* x_ref;
  const float* u_ref;
  const float* u_min;  // device [4] or null (no box)
  const float* u_max;
  int64_t B;
  int T;
  float dt;
  int max_iter;
  float reg;
  float tol;
  int n_alpha;
  float alphas[ILQR_MAX_ALPHAS_DEV];
  int64_t cost_bstride;  // steps between elements in C, c (T batch-major, 1 time-major)
  int64_t cost_tstride;  // steps between time steps (1 batch-major, B time-major)
  const int8_t* forced;  // [B][max_iter] decisions to replay, or null
  int forced_stop;       // iterations the batch runs under replay (0: free)
  float* X;
  float* U;
  float* X_lin;
  float* U_lin;
  uint8_t* tight;
  int8_t* trace;
  float* best_cost;
  // workspace
  int32_t* flags;  // [0] stop, [1] converged, [2] iterations run
  float* slots;
  float* gains;
  float* free_mask;
  FmState state;
};

struct FmBackwardParams {
  const float* X;
  const float* U;
  const float* X_lin;
  const float* U_lin;
  const float* C;
  const float* C_final;
  const float* x_ref;
  const float* u_ref;
  const uint8_t* tight;
  const float* grad_X;
  const float* grad_U;
  int64_t B;
  int T;
  float dt;
  float reg;
  int64_t cost_bstride;
  int64_t cost_tstride;
  float* grad_x0;
  float* grad_C;
  float* grad_c;
  float* grad_C_final;
  float* grad_c_final;
  float* grad_x_ref;
  float* grad_u_ref;
  float* gains;  // workspace
};

size_t solve_ws_bytes(int64_t B, int32_t T, int32_t n_alpha);
size_t backward_ws_bytes(int64_t B, int32_t T);
void carve_solve(FmSolveParams& p, void* ws);
cudaError_t launch_solve(FmSolveParams& p, cudaStream_t stream);
cudaError_t launch_backward(FmBackwardParams& p, cudaStream_t stream);
cudaError_t launch_linearize(const float* X, const float* U, int64_t B, int T, float dt, float* A, float* Bm,
                             cudaStream_t stream);
cudaError_t launch_adjoint_lqr(const float* A, const float* Bm, const float* l_xx, const float* l_uu,
                               const float* l_xu, const float* l_x, const float* l_u, const float* l_xxN,
                               const float* l_xN, const uint8_t* tight, int64_t B, int T, float reg, float* K,
                               float* k, float* v0, cudaStream_t stream);
cudaError_t launch_assembly(const float* K, const float* k, const float* v0, const float* A, const float* Bm,
                            const float* X, const float* U, const float* x_ref, const float* u_ref, int64_t B,
                            int T, float* gC, float* gc, float* gx0, float* gxr, float* gur, float* gCf, float* gcf,
                            cudaStream_t stream);

}  // namespace fm

}  // namespace ilqr
