// Companion kernels of the solver loop: the convergence measures of src/trnopt/sinkhorn.py:358-374.
// One CTA of 1024 threads each: the vectors are at most a few hundred thousand floats, and a single CTA gives a
// deterministic reduction order (the result is compared against a tolerance every check_every iterations).
#include "common.cuh"
#include "kernels.h"

namespace trnopt {

constexpr int RED_THREADS = 1024;

__device__ __forceinline__ double block_sum(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  v = lane < (blockDim.x >> 5) ? sh[lane] : 0.0;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  v = lane < (blockDim.x >> 5) ? sh[lane] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// sum_j | w_j * (exp(min((old_j - new_j) * inv_eps, 50)) - 1) |  (sinkhorn.py:370-371)
__global__ void __launch_bounds__(RED_THREADS) balanced_error_kernel(const float* __restrict__ gh_old,
                                                                     const float* __restrict__ gh_new,
                                                                     const float* __restrict__ w, int n,
                                                                     float inv_eps, float* out) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int j = threadIdx.x; j < n; j += RED_THREADS) {
    const float delta = fminf((gh_old[j] - gh_new[j]) * inv_eps, 50.0f);
    acc += fabs((double)w[j] * ((double)expf(delta) - 1.0));
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) out[0] = (float)acc;
}

// max_j |new_j - old_j| * inv_eps  (sinkhorn.py:360, 373)
__global__ void __launch_bounds__(RED_THREADS) max_change_kernel(const float* __restrict__ gh_old,
                                                                 const float* __restrict__ gh_new, int n,
                                                                 float inv_eps, float* out) {
  __shared__ float sh[32];
  float m = 0.f;
  for (int j = threadIdx.x; j < n; j += RED_THREADS) m = fmaxf(m, fabsf(gh_new[j] - gh_old[j]));
  m = block_max(m, sh);
  if (threadIdx.x == 0) out[0] = m * inv_eps;
}

cudaError_t balanced_error_launch(const float* gh_old, const float* gh_new, const float* w, int n, float inv_eps,
                                  float* out, cudaStream_t stream) {
  balanced_error_kernel<<<1, RED_THREADS, 0, stream>>>(gh_old, gh_new, w, n, inv_eps, out);
  return cudaGetLastError();
}

cudaError_t max_change_launch(const float* gh_old, const float* gh_new, int n, float inv_eps, float* out,
                              cudaStream_t stream) {
  max_change_kernel<<<1, RED_THREADS, 0, stream>>>(gh_old, gh_new, n, inv_eps, out);
  return cudaGetLastError();
}

}  // namespace trnopt
