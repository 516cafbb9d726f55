// ilqr_noalloc.cu -- the solve entry point for callers that cannot allocate
// device memory.
//
// Some hosts must not allocate GPU memory once they are running: a flight or
// robot control loop whose memory budget is fixed at start-up (allocation at
// run time would break its timing guarantees), or a plugin whose host owns
// the device allocator and gives plugins no way to call it. Such a caller
// still owns its inputs and outputs, but cannot hand the solver a workspace.
// ilqr_b200_solve_f32_noalloc runs the same solve as ilqr_b200_solve_f32 with
// its scratch in a fixed array that lives in this library's device image.
//
// The array is a file-scope __device__ variable of ILQR_NOALLOC_SCRATCH_BYTES
// (16 MiB): every GPU that loads this library holds it until the process
// exits. Host code cannot use the array's name as a device address (in host
// code that name denotes a host-side stand-in); its device address is looked
// up once per device with cudaGetSymbolAddress, with that device current,
// the first time the entry point is called on it. That first call should
// therefore come before any stream capture.
#include <mutex>

#include "ilqr_b200.h"

namespace {

constexpr size_t kScratchFloats = ILQR_NOALLOC_SCRATCH_BYTES / sizeof(float);
__device__ __align__(256) float g_solve_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
float* g_scratch_ptr[kMaxDevices];
cudaError_t g_scratch_err[kMaxDevices];

// Device address of the scratch array on the current device (looked up once).
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ILQR_ERR_CUDA;
  std::call_once(g_once[dev], [dev] {
    void* p = nullptr;
    g_scratch_err[dev] = cudaGetSymbolAddress(&p, g_solve_scratch);
    g_scratch_ptr[dev] = static_cast<float*>(p);
  });
  if (g_scratch_err[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr) return ILQR_ERR_CUDA;
  *out = g_scratch_ptr[dev];
  return ILQR_OK;
}

}  // namespace

extern "C" int ilqr_b200_solve_f32_noalloc(
    const float* x0, const float* U_init, const float* C, const float* c, const float* C_final,
    const float* c_final, const float* x_ref, const float* u_ref, const float* u_min, const float* u_max,
    int64_t B, int32_t T, float dt, int32_t max_iter, float reg_eps, float converge_tol, const float* alphas,
    int32_t n_alpha, const int8_t* forced_trace, float* X, float* U, uint8_t* tight_mask, int8_t* trace,
    int32_t* iters, uint32_t* elem_status, float* best_cost, int32_t* stall_iter, float* stall_gap,
    cudaStream_t stream) {
  size_t need = 0;
  const int q = ilqr_b200_solve_workspace_size(B, T, &need);
  if (q != ILQR_OK) return q;
  if (need > ILQR_NOALLOC_SCRATCH_BYTES) return ILQR_ERR_NOALLOC_LIMIT;
  float* scratch = nullptr;
  if (B > 0) {
    const int st = scratch_for_current_device(&scratch);
    if (st != ILQR_OK) return st;
  }
  // The solve writes every scratch word it reads (trajectories by the first
  // rollout, gains by each Riccati pass), so nothing needs clearing between
  // calls even though the array keeps the previous call's contents.
  return ilqr_b200_solve_f32(x0, U_init, C, c, C_final, c_final, x_ref, u_ref, u_min, u_max, B, T, dt,
                             max_iter, reg_eps, converge_tol, alphas, n_alpha, forced_trace, X, U, tight_mask,
                             trace, iters, elem_status, best_cost, stall_iter, stall_gap, scratch,
                             ILQR_NOALLOC_SCRATCH_BYTES, stream);
}
