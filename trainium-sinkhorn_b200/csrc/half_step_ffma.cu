// Fused Sinkhorn half-step, FP32 FFMA tile path (sm_100a).
//
// One CTA of 256 threads computes 128 x 128 score tiles in registers (8 x 8 per thread) from transposed point
// tiles staged in shared memory with cp.async (the column tile double-buffered), adds the per-column bias
// gh_j / eps + log b_j in FP32, and folds each tile into a per-row online (max, sum) in base 2. Scores never
// leave registers. Work is split stream-K style over (row tile, column tile) units; see common.cuh.
//
// This is the plain FP32 path of the reference's half-step (src/trnopt/sinkhorn.py:108-119); the tensor-core
// path is half_step_tc.cu. It is also the path for the row-LSE entry point (the quantity of
// src/trnopt/nki_sinkhorn.py:150-172).
#include "common.cuh"
#include "kernels.h"

namespace trnopt {

constexpr int FF_BM = 128;
constexpr int FF_BN = 128;
constexpr int FF_THREADS = 256;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// dst[k * 128 + j] = src[k * ld + c0 + j] for k < d, j < 128; zero where c0 + j >= limit.
// Requires ld % 4 == 0 and a 16-byte aligned src (checked by the host API).
__device__ __forceinline__ void load_tile_async(float* dst, const float* src, int ld, int c0, int limit, int d,
                                                int tid) {
  const int chunks = d * 32;
  for (int q = tid; q < chunks; q += FF_THREADS) {
    const int k = q >> 5, j4 = (q & 31) * 4;
    const int col = c0 + j4;
    int valid = limit - col;
    valid = valid < 0 ? 0 : (valid > 4 ? 4 : valid);
    const float* g = src + (size_t)k * ld + (valid > 0 ? col : 0);
    cp_async16(dst + k * 128 + j4, g, valid * 4);
  }
}

__device__ __forceinline__ void load_bias(float* dst, const LseProblem& p, int c0, int tid) {
  if (tid < FF_BN) {
    const int j = c0 + tid;
    float b = -INFINITY;
    if (j < p.m) {
      b = 0.f;
      if (p.gh) b = p.gh[j] * p.gh2;
      if (p.log_b) b = fmaf(p.log_b[j], p.lb2, b);
    }
    dst[tid] = b;
  }
}

__global__ void __launch_bounds__(FF_THREADS, 2) lse_ffma_kernel(LseProblem p, StreamK sk) {
  if (p.dyn != nullptr) {
    // a run decided on the device: eps and kappa of the state's current stage; nothing to do once it is done
    const TrnoptSolveState* st = p.dyn;
    if (st->done) return;
    p.dot2 = st->dot2;
    p.gh2 = st->gh2;
    p.eps = (double)st->eps;
    p.kappa = (double)st->kappa[p.side];
  }
  extern __shared__ __align__(16) float smem[];
  __shared__ int s_last;
  const int d = p.d;
  float* xs = smem;                 // [d][128]
  float* ys = xs + d * FF_BM;       // [2][d][128]
  float* bs = ys + 2 * d * FF_BN;   // [2][128]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

  const long long u_end = sk_unit_begin(blockIdx.x + 1, sk.units, sk.grid);
  long long u = sk_unit_begin(blockIdx.x, sk.units, sk.grid);
  while (u < u_end) {
    const int r = (int)(u / sk.nct);
    const int c_first = (int)(u % sk.nct);
    const long long seg_end = min(u_end, (long long)(r + 1) * sk.nct);
    const int ntile = (int)(seg_end - u);
    const int r0 = r * FF_BM;

    __syncthreads();                                       // the previous segment is done with all buffers
    load_tile_async(xs, p.xT, p.ldx, r0, p.rows, d, tid);
    cp_async_commit();
    load_tile_async(ys, p.yT, p.ldy, c_first * FF_BN, p.m, d, tid);
    load_bias(bs, p, c_first * FF_BN, tid);
    cp_async_commit();

    float M[8], L[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { M[i] = kMaxFloor; L[i] = 0.f; }

    for (int t = 0; t < ntile; ++t) {
      const int buf = t & 1;
      if (t + 1 < ntile) {
        const int c1 = (c_first + t + 1) * FF_BN;
        load_tile_async(ys + (buf ^ 1) * d * FF_BN, p.yT, p.ldy, c1, p.m, d, tid);
        load_bias(bs + (buf ^ 1) * FF_BN, p, c1, tid);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();

      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
      const float* yb = ys + buf * d * FF_BN;
#pragma unroll 4
      for (int k = 0; k < d; ++k) {
        const float4 a0 = *reinterpret_cast<const float4*>(xs + k * FF_BM + ty * 4);
        const float4 a1 = *reinterpret_cast<const float4*>(xs + k * FF_BM + 64 + ty * 4);
        const float4 b0 = *reinterpret_cast<const float4*>(yb + k * FF_BN + tx * 4);
        const float4 b1 = *reinterpret_cast<const float4*>(yb + k * FF_BN + 64 + tx * 4);
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }

      const float* bias = bs + buf * FF_BN;
      float bj[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) { bj[q] = bias[tx * 4 + q]; bj[4 + q] = bias[64 + tx * 4 + q]; }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float tv[8];
        float tmax = kMaxFloor;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          tv[j] = fmaf(acc[i][j], p.dot2, bj[j]);
          tmax = fmaxf(tmax, tv[j]);
        }
        if (tmax > M[i]) {
          L[i] *= ex2_approx(M[i] - tmax);
          M[i] = tmax;
        }
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) s += ex2_approx(tv[j] - M[i]);
        L[i] += s;
      }
      __syncthreads();                                     // everyone is done reading buffer `buf`
    }

    // Merge the 16 column groups of each row (lanes tx = 0..15 of a half warp).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        const float M2 = __shfl_xor_sync(0xffffffffu, M[i], o);
        const float L2 = __shfl_xor_sync(0xffffffffu, L[i], o);
        lse_merge(M[i], L[i], M2, L2);
      }
    }
    const long long first_u = (long long)r * sk.nct;
    const int kfirst = sk_cta_of(first_u, sk.units, sk.grid);
    const int klast = sk_cta_of(first_u + sk.nct - 1, sk.units, sk.grid);
    const int expected = klast - kfirst + 1;
    float2* part = sk.partials + ((size_t)r * sk.slots + (blockIdx.x - kfirst)) * FF_BM;
    if (tx == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        part[ty * 4 + q] = make_float2(M[q], L[q]);
        part[64 + ty * 4 + q] = make_float2(M[4 + q], L[4 + q]);
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(&sk.counters[r], 1);
      s_last = (old == expected - 1);
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tid < FF_BM && r0 + tid < p.rows)
        finish_row(p, r0 + tid, sk.partials + (size_t)r * sk.slots * FF_BM + tid, expected, FF_BM, p.eps, p.kappa);
      if (tid == 0) sk.counters[r] = 0;
    }
    u = seg_end;
  }
}

size_t ffma_smem_bytes(int d) { return (size_t)(3 * d * 128 + 2 * 128) * sizeof(float); }

int ffma_grid(int device, int d, long long units) {
  // Per device: SM count, the shared-memory opt-in (one for the largest tile, d = 128: the attribute is a ceiling,
  // every launch asks for its own size) and the resident blocks per SM for each d.
  static std::atomic<int> sms[kMaxDevices], attr_done[kMaxDevices];
  static std::atomic<int> blocks_for[kMaxDevices][129];
  if (device < 0 || device >= kMaxDevices) device = 0;
  int n_sm = sms[device].load();
  if (n_sm == 0) {
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device);
    sms[device].store(n_sm);
  }
  smem_attr_once(reinterpret_cast<const void*>(lse_ffma_kernel), (int)ffma_smem_bytes(128), attr_done);
  int blocks = blocks_for[device][d].load();
  if (blocks == 0) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, lse_ffma_kernel, FF_THREADS, ffma_smem_bytes(d));
    blocks = blocks > 0 ? blocks : 1;
    blocks_for[device][d].store(blocks);
  }
  long long g = (long long)blocks * (n_sm > 0 ? n_sm : 148);
  return (int)(g < units ? g : units);
}

void ffma_plan(int device, int rows, int m, int d, StreamK& sk) {
  sk.nrt = (rows + FF_BM - 1) / FF_BM;
  sk.nct = (m + FF_BN - 1) / FF_BN;
  sk.units = (long long)sk.nrt * sk.nct;
  sk.grid = ffma_grid(device, d, sk.units);
  sk.slots = sk_max_slots(sk.units, sk.grid, sk.nct);
  sk.parts_per_cta = 1;
}

size_t ffma_partial_bytes(const StreamK& sk) { return (size_t)sk.nrt * sk.slots * FF_BM * sizeof(float2); }

cudaError_t ffma_launch(const LseProblem& p, const StreamK& sk, cudaStream_t stream) {
  const size_t smem = ffma_smem_bytes(p.d);
  lse_ffma_kernel<<<sk.grid, FF_THREADS, smem, stream>>>(p, sk);
  return cudaGetLastError();
}

}  // namespace trnopt
