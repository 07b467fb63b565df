// Internal declarations shared between the kernel files and the C-ABI layer (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include <atomic>

#include "common.cuh"

namespace trnopt {

constexpr int kMaxDevices = 64;

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) acts on the calling thread's current device only. `done` holds,
// per device, the largest size already set for `fn`, so a process that drives several GPUs sets it on each of them.
inline cudaError_t smem_attr_once(const void* fn, int bytes, std::atomic<int>* done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    int cur = done[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !done[dev].compare_exchange_weak(cur, bytes, std::memory_order_release)) {
    }
  }
  return e;
}

// FFMA tile path (half_step_ffma.cu)
size_t ffma_smem_bytes(int d);
void ffma_plan(int device, int rows, int m, int d, StreamK& sk);
size_t ffma_partial_bytes(const StreamK& sk);
cudaError_t ffma_launch(const LseProblem& p, const StreamK& sk, cudaStream_t stream);

// tcgen05 split-precision path (half_step_tc.cu)
struct TcProblem;
int tc_supported_d(int d);                       // packed K per half (16-element multiple), 0 if unsupported
int tc_kp(int d);                                // FP16 elements per packed row
void tc_plan(int device, int rows, int m, int d, StreamK& sk);
size_t tc_partial_bytes(const StreamK& sk);
cudaError_t tc_pack(const float* xT, int ldx, int n, int d, int scale_exp, void* packed, cudaStream_t stream);
cudaError_t tc_launch(const LseProblem& p, const void* xpack, const void* ypack, int sx, int sy, const StreamK& sk,
                      cudaStream_t stream, const Publish* pub = nullptr, bool pdl = true);

// companions (companions.cu)
cudaError_t balanced_error_launch(const float* gh_old, const float* gh_new, const float* w, int n, float inv_eps,
                                  float* out, cudaStream_t stream);
cudaError_t recenter_launch(float* gh, int n, int npad, double* gauge, const TrnoptSolveState* st,
                            cudaStream_t stream);
cudaError_t max_change_launch(const float* gh_old, const float* gh_new, int n, float inv_eps, float* out,
                              cudaStream_t stream);

// exact median of all clamped costs (median.cu)
size_t median_workspace_bytes();
cudaError_t median_launch(const double* x, const double* y, const double* sqx, const double* sqy, int n, int m,
                          int d, double* out, void* ws, cudaStream_t stream);

// plan evaluation from potentials, float64 (plan.cu)
int plan_lse_splits(int device, int n, int m);
size_t plan_lse_workspace_bytes(int device, int n, int m);
cudaError_t plan_rows_launch(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                             const double* la, const double* lb, double eps, const int* rows, int nrows, double* out,
                             cudaStream_t stream);
cudaError_t plan_lse_launch(int device, const double* x, int n, const double* y, int m, int d, const double* f,
                            const double* g, const double* la, const double* lb, double eps, double* out, void* ws,
                            cudaStream_t stream);

cudaError_t ex2_poly_launch(const float* x, float* out, int n, cudaStream_t stream);

int* device_error_word();

// Argument checks of the tcgen05 half-step (pointers, sizes, 128-byte packed clouds, finite eps > 0 and kappa, a
// compute capability 10 device); TRNOPT_OK or the status trnopt_half_step_tc returns for them. Enqueues nothing.
int half_step_tc_check(const void* xpack, const float* xsq, const void* ypack, const float* gh, const float* log_b,
                       int rows, int m, int d, float eps, float kappa, const float* fh);

// The tcgen05 half-step behind trnopt_half_step_tc, with an optional Publish (capi.cu); returns a TRNOPT status.
int half_step_tc_launch(const void* xpack, const float* xsq, const float* off, const void* ypack, const float* gh,
                        const float* log_b, int rows, int m, int d, int sx, int sy, float eps, float kappa, float* fh,
                        void* workspace, size_t ws_bytes, cudaStream_t stream, const Publish* pub,
                        const TrnoptSolveState* dyn = nullptr, int side = 0, bool pdl = true);

// The FFMA half-step behind trnopt_half_step, optionally reading its scalars from a solve state (capi.cu).
int half_step_ffma_launch(const float* xT, int ldx, const float* xsq, const float* off, const float* yT, int ldy,
                          const float* gh, const float* log_b, int rows, int m, int d, float eps, float kappa, float* fh,
                          void* workspace, size_t ws_bytes, cudaStream_t stream, const TrnoptSolveState* dyn,
                          int side);

// The solver loop's check after a run of n iterations (companions.cu): advances the state's counters and applies
// the reference loop's stage and convergence rules.
cudaError_t solve_check_launch(TrnoptSolveState* st, int n, const float* g0, const float* g1, const float* w,
                               cudaStream_t stream);
// A stage's half-step parameters, computed as a host call computes them (float eps, float kappa, float dot2 / gh2).
__host__ __device__ inline void solve_stage_params(TrnoptSolveState& st) {
  const int s = st.stage < st.n_stages ? st.stage : st.n_stages;
  const double e = st.stage_eps[s];
  st.eps = (float)e;
  const double inv = 1.0 / (double)st.eps;
  st.dot2 = (float)(2.0 * inv * 1.4426950408889634);
  st.gh2 = (float)(inv * 1.4426950408889634);
  for (int k = 0; k < 2; ++k) st.kappa[k] = st.rho[k] < 0.0 ? 1.0f : (float)(st.rho[k] / (st.rho[k] + e));
}

}  // namespace trnopt
