// Exact median of all n * m clamped squared-distance costs, for the "median" cost normalization of trnopt
// (reference src/trnopt/sinkhorn.py:229-233, used once per pair by src/trnopt/singlecell.py:72).
//
// The reference builds the whole n x m cost matrix in float64 on the host,
//     C = (|xc|^2[:, None] + |yc|^2[None, :]) - 2.0 * (xc @ yc.T),   scale = median(max(C, 0)),
// and np.median averages the two middle order statistics when n m is even. Here no cost is ever stored: a radix
// select over the 64-bit patterns of the (non-negative) float64 costs runs 8 passes of 8 bits; each pass
// re-evaluates the costs tile by tile in float64 (same expression and association as the reference, FMA
// contraction off for the final combination) and histograms the next digit of the costs whose higher digits match
// the prefix found so far. A one-thread kernel between passes picks the bucket holding the wanted rank. The
// squared norms |xc|^2, |yc|^2 come from the host (numpy, as the reference computes them).
#include "common.cuh"
#include "kernels.h"

namespace trnopt {

constexpr int MD_TILE = 64;
constexpr int MD_THREADS = 256;

struct MedianState {
  unsigned long long prefix;   // digits found so far (higher bits of the wanted key)
  unsigned long long rank;     // rank of the wanted key among the keys that match the prefix
  unsigned long long key[2];   // results of the two selections
};

__device__ __forceinline__ unsigned long long cost_key(double c) {
  // max(C, 0): negative costs (and -0.0) become +0.0; non-negative doubles order like their bit patterns.
  return c > 0.0 ? (unsigned long long)__double_as_longlong(c) : 0ull;
}

__global__ void __launch_bounds__(MD_THREADS) median_hist_kernel(const double* __restrict__ x,
                                                                 const double* __restrict__ y,
                                                                 const double* __restrict__ sqx,
                                                                 const double* __restrict__ sqy, int n, int m,
                                                                 int d, const MedianState* __restrict__ st,
                                                                 unsigned* __restrict__ hist, int pass) {
  extern __shared__ __align__(16) double msm[];
  __shared__ unsigned h[256];
  double* xs = msm;                 // [d][64]
  double* ys = msm + d * MD_TILE;   // [d][64]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nct = (m + MD_TILE - 1) / MD_TILE;
  const int r0 = (int)(blockIdx.x / nct) * MD_TILE, c0 = (int)(blockIdx.x % nct) * MD_TILE;
  h[tid] = 0;
  for (int q = tid; q < d * MD_TILE; q += MD_THREADS) {
    const int i = q / d, k = q % d;
    xs[k * MD_TILE + i] = (r0 + i < n) ? x[(size_t)(r0 + i) * d + k] : 0.0;
    ys[k * MD_TILE + i] = (c0 + i < m) ? y[(size_t)(c0 + i) * d + k] : 0.0;
  }
  __syncthreads();
  double acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.0;
  for (int k = 0; k < d; ++k) {
    double xa[4], yb[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) xa[a] = xs[k * MD_TILE + ty + 16 * a];
#pragma unroll
    for (int b = 0; b < 4; ++b) yb[b] = ys[k * MD_TILE + tx + 16 * b];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fma(xa[a], yb[b], acc[a][b]);
  }
  const int shift = 56 - 8 * pass;
  const unsigned long long prefix = st->prefix;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int i = r0 + ty + 16 * a;
    if (i >= n) continue;
    const double sx = sqx[i];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int j = c0 + tx + 16 * b;
      if (j >= m) continue;
      const double c = __dsub_rn(__dadd_rn(sx, sqy[j]), __dmul_rn(2.0, acc[a][b]));
      const unsigned long long key = cost_key(c);
      if (pass == 0 || (key >> (shift + 8)) == (prefix >> (shift + 8)))
        atomicAdd(&h[(unsigned)(key >> shift) & 255u], 1u);
    }
  }
  __syncthreads();
  if (h[tid]) atomicAdd(&hist[tid], h[tid]);
}

// Pick the bucket that holds st->rank, extend the prefix, rebase the rank, clear the histogram.
__global__ void median_select_kernel(MedianState* st, unsigned* hist, int pass, int which) {
  if (threadIdx.x != 0) return;
  const int shift = 56 - 8 * pass;
  unsigned long long r = st->rank, before = 0;
  int b = 0;
  for (; b < 255; ++b) {
    if (before + hist[b] > r) break;
    before += hist[b];
  }
  st->prefix |= (unsigned long long)b << shift;
  st->rank = r - before;
  for (int i = 0; i < 256; ++i) hist[i] = 0;
  if (pass == 7) st->key[which] = st->prefix;
}

__global__ void median_init_kernel(MedianState* st, unsigned* hist, unsigned long long rank) {
  if (threadIdx.x == 0) {
    st->prefix = 0;
    st->rank = rank;
  }
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
}

__global__ void median_finish_kernel(const MedianState* st, int two, double* out) {
  const double a = __longlong_as_double((long long)st->key[0]);
  if (!two) {
    out[0] = a;
  } else {
    const double b = __longlong_as_double((long long)st->key[1]);
    out[0] = (a + b) / 2.0;       // np.median: mean of the two middle values
  }
}

size_t median_workspace_bytes() { return sizeof(MedianState) + 256 * sizeof(unsigned) + 256; }

cudaError_t median_launch(const double* x, const double* y, const double* sqx, const double* sqy, int n, int m,
                          int d, double* out, void* ws, cudaStream_t stream) {
  MedianState* st = reinterpret_cast<MedianState*>(ws);
  unsigned* hist = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(ws) + 256);
  const unsigned long long N = (unsigned long long)n * (unsigned long long)m;
  const int two = (N % 2ull) == 0ull;
  const unsigned long long ranks[2] = {two ? N / 2 - 1 : N / 2, N / 2};
  const size_t smem = (size_t)2 * d * MD_TILE * sizeof(double);
  static std::atomic<int> attr_done[kMaxDevices];
  cudaError_t e = smem_attr_once(reinterpret_cast<const void*>(median_hist_kernel), (int)smem, attr_done);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)(((m + MD_TILE - 1) / MD_TILE) * (long long)((n + MD_TILE - 1) / MD_TILE));
  for (int w = 0; w < 1 + two; ++w) {
    median_init_kernel<<<1, 256, 0, stream>>>(st, hist, ranks[w]);
    for (int pass = 0; pass < 8; ++pass) {
      median_hist_kernel<<<grid, MD_THREADS, smem, stream>>>(x, y, sqx, sqy, n, m, d, st, hist, pass);
      median_select_kernel<<<1, 32, 0, stream>>>(st, hist, pass, w);
    }
  }
  median_finish_kernel<<<1, 1, 0, stream>>>(st, two, out);
  return cudaGetLastError();
}

}  // namespace trnopt
