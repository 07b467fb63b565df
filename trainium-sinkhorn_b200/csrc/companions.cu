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

// sum_j | w_j * (exp(min((old_j - new_j) * inv_eps, 50)) - 1) |  (sinkhorn.py:370-371); valid in thread 0.
__device__ __forceinline__ float balanced_error_block(const float* __restrict__ gh_old,
                                                      const float* __restrict__ gh_new, const float* __restrict__ w,
                                                      int n, float inv_eps, double* sh) {
  double acc = 0.0;
  for (int j = threadIdx.x; j < n; j += RED_THREADS) {
    const float delta = fminf((gh_old[j] - gh_new[j]) * inv_eps, 50.0f);
    acc += fabs((double)w[j] * ((double)expf(delta) - 1.0));
  }
  return (float)block_sum(acc, sh);
}

// max_j |new_j - old_j| * inv_eps  (sinkhorn.py:360, 373); valid in thread 0.
__device__ __forceinline__ float max_change_block(const float* __restrict__ gh_old, const float* __restrict__ gh_new,
                                                  int n, float inv_eps, float* sh) {
  float m = 0.f;
  for (int j = threadIdx.x; j < n; j += RED_THREADS) m = fmaxf(m, fabsf(gh_new[j] - gh_old[j]));
  return block_max(m, sh) * inv_eps;
}

__global__ void __launch_bounds__(RED_THREADS) balanced_error_kernel(const float* __restrict__ gh_old,
                                                                     const float* __restrict__ gh_new,
                                                                     const float* __restrict__ w, int n,
                                                                     float inv_eps, float* out) {
  __shared__ double sh[32];
  const float e = balanced_error_block(gh_old, gh_new, w, n, inv_eps, sh);
  if (threadIdx.x == 0) out[0] = e;
}

__global__ void __launch_bounds__(RED_THREADS) max_change_kernel(const float* __restrict__ gh_old,
                                                                 const float* __restrict__ gh_new, int n,
                                                                 float inv_eps, float* out) {
  __shared__ float sh[32];
  const float m = max_change_block(gh_old, gh_new, n, inv_eps, sh);
  if (threadIdx.x == 0) out[0] = m;
}

// The solver loop's decisions after a run of n iterations (the reference's loop, sinkhorn.py:346-378, at the run's
// last iteration, where a check falls): the counters advance by n; inside an intermediate eps stage a check every
// check_every iterations of the stage compares the maximum potential change with the stage tolerance (or the
// stage's iteration limit) and moves on to the next stage; at the final eps, unless fixed_iters, a check every
// check_every iterations (and at max_iters) computes the balanced marginal error or the maximum change and ends the
// solve below tol. The potentials before and after the run's last iteration are G[(it - 1) % 2] and G[it % 2].
__global__ void __launch_bounds__(RED_THREADS) solve_check_kernel(TrnoptSolveState* st, int n,
                                                                  const float* __restrict__ g0,
                                                                  const float* __restrict__ g1,
                                                                  const float* __restrict__ w) {
  __shared__ double shd[32];
  __shared__ float shf[32];
  if (st->done) return;                                     // uniform: the state is not written during this kernel
  const int it = st->it + n, stage_it = st->stage_it + n, stage = st->stage;
  const float* gh_prev = ((it - 1) & 1) ? g1 : g0;
  const float* gh_new = (it & 1) ? g1 : g0;
  const int s = stage < st->n_stages ? stage : st->n_stages;
  const float inv_eps = (float)(1.0 / st->stage_eps[s]);
  const bool in_stage = stage < st->n_stages;
  bool check, use_balanced = false;
  if (in_stage) {
    check = stage_it % st->check_every == 0;
  } else {
    check = !st->fixed_iters && (st->n_stages > 0 || it > st->sched_len) &&
            (stage_it % st->check_every == 0 || it == st->max_iters);
    use_balanced = st->balanced != 0;
  }
  float v = 0.f;
  if (check) v = use_balanced ? balanced_error_block(gh_prev, gh_new, w, st->npad, inv_eps, shd)
                              : max_change_block(gh_prev, gh_new, st->n_real, inv_eps, shf);
  if (threadIdx.x != 0) return;
  st->it = it;
  st->stage_it = stage_it;
  if (in_stage) {
    if (check && (v < st->stage_tol || stage_it >= st->stage_max_iters)) {
      st->stage_iters[stage] = stage_it;
      st->stage = stage + 1;
      st->stage_it = 0;
      solve_stage_params(*st);
    }
  } else if (check) {
    st->err = v;
    if (v < st->tol) {
      st->converged = 1;
      st->done = 1;
    }
  }
  if (it >= st->max_iters) st->done = 1;
}

cudaError_t solve_check_launch(TrnoptSolveState* st, int n, const float* g0, const float* g1, const float* w,
                               cudaStream_t stream) {
  solve_check_kernel<<<1, RED_THREADS, 0, stream>>>(st, n, g0, g1, w);
  return cudaGetLastError();
}

// Balanced solves keep the potential they iterate on near zero. (f + c, g - c) gives the same plan, and in exact
// arithmetic the iteration carries a constant c through unchanged, but the reference's starting point leaves a large
// constant in the shifted potentials (about 21 on config 2, against a spread of 0.4), where float32 storage and the
// float32 scores lose 5 bits; the rounding error then repeats almost identically every iteration near convergence and
// adds up along the slowest mode. This kernel moves the input potential of a run by K = its mean over the n real
// points, rounded to float32 (gh -= K on all npad entries: exact by Sterbenz' lemma wherever gh lies within a factor 2
// of K), and adds K to the float64 offset that the final unshift puts back (g + K, f - K), so the returned potentials
// are the reference's. Deterministic (fixed reduction order).
__global__ void __launch_bounds__(RED_THREADS) recenter_kernel(float* __restrict__ gh, int n, int npad,
                                                               double* __restrict__ gauge,
                                                               const TrnoptSolveState* st) {
  __shared__ double sh[32];
  __shared__ float s_k;
  if (st != nullptr && st->done) return;
  double acc = 0.0;
  for (int j = threadIdx.x; j < n; j += RED_THREADS) acc += (double)gh[j];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) {
    const float k = (float)(acc / (double)n);
    s_k = k;
    gauge[0] += (double)k;
  }
  __syncthreads();
  const float k = s_k;
  for (int j = threadIdx.x; j < npad; j += RED_THREADS) gh[j] -= k;
}

cudaError_t recenter_launch(float* gh, int n, int npad, double* gauge, const TrnoptSolveState* st,
                            cudaStream_t stream) {
  recenter_kernel<<<1, RED_THREADS, 0, stream>>>(gh, n, npad, gauge, st);
  return cudaGetLastError();
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
