// Internal declarations shared between the kernel files and the C-ABI layer (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "common.cuh"

namespace trnopt {

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
                      cudaStream_t stream);

// companions (companions.cu)
cudaError_t balanced_error_launch(const float* gh_old, const float* gh_new, const float* w, int n, float inv_eps,
                                  float* out, cudaStream_t stream);
cudaError_t max_change_launch(const float* gh_old, const float* gh_new, int n, float inv_eps, float* out,
                              cudaStream_t stream);

// exact median of all clamped costs (median.cu)
size_t median_workspace_bytes();
cudaError_t median_launch(const double* x, const double* y, const double* sqx, const double* sqy, int n, int m,
                          int d, double* out, void* ws, cudaStream_t stream);

cudaError_t ex2_poly_launch(const float* x, float* out, int n, cudaStream_t stream);

int* device_error_word();

}  // namespace trnopt
