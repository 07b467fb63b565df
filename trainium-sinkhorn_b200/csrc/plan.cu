// On-demand evaluation of the transport plan from converged potentials, in float64, without building the dense
// n x m matrix on the host:
//     P_ij = exp(log_a_i + log_b_j + (f_i + g_j - C_ij) / eps),   C_ij = sum_k (x_ik - y_jk)^2
// This is the plan of the reference's transport_plan (src/trnopt/sinkhorn.py:397-403) with its direct-difference
// cost. Two kernels share one 64 x 64 cost tile (C for 64 rows of x and 64 rows of y, coordinates staged through
// shared memory 32 at a time, each of 256 threads holding a 4 x 4 block of the tile):
//   plan_rows        the full rows P_{r,:} for a list of row indices r (transport_plan / wot_tmap row by row,
//                    src/trnopt/singlecell.py:89-92);
//   plan_lse         out_i = log sum_j P_ij, per-(row, column split) partial (max, sum) pairs merged by a second
//                    kernel in a fixed order (deterministic). With x and y swapped it gives log column sums, so
//                    it serves the plan marginals of examples/sinkhorn_libs_compare.py:43-56 and, with log_a = 0
//                    and log_b = log v, the ancestor pull-back log(P v) of examples/singlecell_figures.py:35-47.
// All work is float64 (the reference evaluates these on the host in float64); the kernels are bound by the FP64
// pipe: 2 FP64 operations per (i, j, k) plus one exp per (i, j).
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace trnopt {

constexpr int PT = 64;        // tile rows = tile columns
constexpr int PKC = 32;       // coordinates staged per pass
constexpr int PTHREADS = 256;
constexpr int PPAD = PT + 1;  // padded smem rows: staging stores hit 2 banks per pair, not 32

struct PlanSmem {
  double xs[PKC][PPAD];
  double ys[PKC][PPAD];
  int xi[PT];  // global row index of each tile row, -1 outside
  int yj[PT];  // global column index of each tile column, -1 outside
};

// C for the CTA's tile: thread (tr, tc) = (t / 16, t % 16) owns rows tr + 16 a and columns tc + 16 b (a, b < 4).
// s.xi / s.yj must be set and visible (after a __syncthreads) before the call; returns with all threads past the
// last read of s.xs / s.ys only after the caller's next __syncthreads.
__device__ __forceinline__ void cost_tile(PlanSmem& s, const double* __restrict__ x, const double* __restrict__ y,
                                          int d, double (&c)[4][4]) {
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) c[a][b] = 0.0;
  for (int k0 = 0; k0 < d; k0 += PKC) {
    const int kc = min(PKC, d - k0);
    __syncthreads();  // previous chunk fully consumed
    for (int q = t; q < PT * PKC; q += PTHREADS) {
      const int r = q / PKC, kk = q % PKC;
      const int i = s.xi[r], j = s.yj[r];
      s.xs[kk][r] = (i >= 0 && kk < kc) ? x[(size_t)i * d + k0 + kk] : 0.0;
      s.ys[kk][r] = (j >= 0 && kk < kc) ? y[(size_t)j * d + k0 + kk] : 0.0;
    }
    __syncthreads();
    for (int kk = 0; kk < kc; ++kk) {
      double xv[4], yv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xv[a] = s.xs[kk][tr + 16 * a];
#pragma unroll
      for (int b = 0; b < 4; ++b) yv[b] = s.ys[kk][tc + 16 * b];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const double u = xv[a] - yv[b];
          c[a][b] = fma(u, u, c[a][b]);
        }
    }
  }
}

__device__ __forceinline__ double opt_load(const double* p, int i) { return p ? p[i] : 0.0; }

// grid.x = ceil(nrows / 64) * ceil(m / 64); out is (nrows, m) row-major. A row index outside [0, n) gives a row of
// NaN (nothing is read for it).
__global__ void __launch_bounds__(PTHREADS) plan_rows_kernel(const double* __restrict__ x, int n,
                                                             const double* __restrict__ y, int m, int d,
                                                             const double* __restrict__ f,
                                                             const double* __restrict__ g,
                                                             const double* __restrict__ la,
                                                             const double* __restrict__ lb, double eps,
                                                             const int* __restrict__ rows, int nrows,
                                                             double* __restrict__ out) {
  __shared__ PlanSmem s;
  const int nct = (m + PT - 1) / PT;
  const int r0 = (int)(blockIdx.x / nct) * PT, c0 = (int)(blockIdx.x % nct) * PT;
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
  if (t < PT) {
    int i = -1;
    if (r0 + t < nrows) {
      i = rows[r0 + t];
      if (i < 0 || i >= n) i = -2;
    }
    s.xi[t] = i < 0 ? -1 : i;
    s.yj[t] = c0 + t < m ? c0 + t : -1;
  }
  __syncthreads();
  double c[4][4];
  cost_tile(s, x, y, d, c);
  __syncthreads();
  double gj[4], lbj[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int j = c0 + tc + 16 * b;
    gj[b] = j < m ? opt_load(g, j) : 0.0;
    lbj[b] = j < m ? opt_load(lb, j) : 0.0;
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int r = r0 + tr + 16 * a;
    if (r >= nrows) continue;
    const int i = s.xi[tr + 16 * a];
    const double fi = i >= 0 ? opt_load(f, i) : 0.0, lai = i >= 0 ? opt_load(la, i) : 0.0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int j = c0 + tc + 16 * b;
      if (j >= m) continue;
      out[(size_t)r * m + j] = i >= 0 ? exp(lai + lbj[b] + (fi + gj[b] - c[a][b]) / eps) : nan("");
    }
  }
}

// Merge of two (max, sum-of-exp(z - max)) pairs; an empty pair has max -inf and sum 0.
__device__ __forceinline__ void lse2_merge(double& M, double& L, double oM, double oL) {
  if (oM == -INFINITY) return;
  if (M == -INFINITY) { M = oM; L = oL; return; }
  if (oM > M) { L = L * exp(M - oM) + oL; M = oM; }
  else L += oL * exp(oM - M);
}

// grid = (ceil(n / 64), splits); CTA (rt, s) covers column tiles [s * nct / splits, (s + 1) * nct / splits) and
// writes, for each of its rows, the pair (max_j z_ij, sum_j exp(z_ij - max)) with
// z_ij = log_b_j + (g_j - C_ij) / eps into pm / pl [s * n + i].
__global__ void __launch_bounds__(PTHREADS) plan_lse_partial_kernel(const double* __restrict__ x, int n,
                                                                    const double* __restrict__ y, int m, int d,
                                                                    const double* __restrict__ g,
                                                                    const double* __restrict__ lb, double inv_eps,
                                                                    double* __restrict__ pm,
                                                                    double* __restrict__ pl) {
  __shared__ PlanSmem s;
  const int nct = (m + PT - 1) / PT, splits = gridDim.y;
  const int r0 = blockIdx.x * PT;
  const int cb = (int)((long long)blockIdx.y * nct / splits), ce = (int)((long long)(blockIdx.y + 1) * nct / splits);
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
  if (t < PT) s.xi[t] = r0 + t < n ? r0 + t : -1;
  double M[4], L[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) { M[a] = -INFINITY; L[a] = 0.0; }
  for (int ct = cb; ct < ce; ++ct) {
    const int c0 = ct * PT;
    __syncthreads();  // previous tile's reads of s.yj done
    if (t < PT) s.yj[t] = c0 + t < m ? c0 + t : -1;
    __syncthreads();
    double c[4][4];
    cost_tile(s, x, y, d, c);
    double bj[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int j = c0 + tc + 16 * b;
      bj[b] = j < m ? opt_load(lb, j) + opt_load(g, j) * inv_eps : -INFINITY;
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      double z[4], mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        z[b] = bj[b] - c[a][b] * inv_eps;
        mx = fmax(mx, z[b]);
      }
      if (mx == -INFINITY) continue;
      if (mx > M[a]) { L[a] = M[a] == -INFINITY ? 0.0 : L[a] * exp(M[a] - mx); M[a] = mx; }
#pragma unroll
      for (int b = 0; b < 4; ++b) L[a] += exp(z[b] - M[a]);
    }
  }
  // the 16 threads sharing tr are 16 consecutive lanes of one warp
#pragma unroll
  for (int a = 0; a < 4; ++a) {
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) {
      const double oM = __shfl_xor_sync(0xffffffffu, M[a], o), oL = __shfl_xor_sync(0xffffffffu, L[a], o);
      lse2_merge(M[a], L[a], oM, oL);
    }
    const int i = r0 + tr + 16 * a;
    if (tc == 0 && i < n) {
      pm[(size_t)blockIdx.y * n + i] = M[a];
      pl[(size_t)blockIdx.y * n + i] = L[a];
    }
  }
}

// out_i = log_a_i + f_i / eps + log sum over splits (in split order); -inf when every term is zero.
__global__ void plan_lse_merge_kernel(const double* __restrict__ pm, const double* __restrict__ pl, int n,
                                      int splits, const double* __restrict__ f, const double* __restrict__ la,
                                      double inv_eps, double* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double M = -INFINITY, L = 0.0;
  for (int s = 0; s < splits; ++s) lse2_merge(M, L, pm[(size_t)s * n + i], pl[(size_t)s * n + i]);
  const double row = opt_load(la, i) + opt_load(f, i) * inv_eps;
  out[i] = M == -INFINITY ? -INFINITY : row + M + log(L);
}

int plan_lse_splits(int device, int n, int m) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const long long rts = (n + PT - 1) / PT, nct = (m + PT - 1) / PT;
  long long s = (2LL * sms + rts - 1) / rts;  // at least two CTAs per SM
  if (s > nct) s = nct;
  if (s > 64) s = 64;
  return (int)(s < 1 ? 1 : s);
}

size_t plan_lse_workspace_bytes(int device, int n, int m) {
  return (size_t)2 * plan_lse_splits(device, n, m) * (size_t)n * sizeof(double);
}

cudaError_t plan_rows_launch(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                             const double* la, const double* lb, double eps, const int* rows, int nrows, double* out,
                             cudaStream_t stream) {
  const long long tiles = (long long)((nrows + PT - 1) / PT) * ((m + PT - 1) / PT);
  if (tiles < 1) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  plan_rows_kernel<<<(unsigned)tiles, PTHREADS, 0, stream>>>(x, n, y, m, d, f, g, la, lb, eps, rows, nrows, out);
  return cudaGetLastError();
}

cudaError_t plan_lse_launch(int device, const double* x, int n, const double* y, int m, int d, const double* f,
                            const double* g, const double* la, const double* lb, double eps, double* out, void* ws,
                            cudaStream_t stream) {
  const int splits = plan_lse_splits(device, n, m);
  double* pm = static_cast<double*>(ws);
  double* pl = pm + (size_t)splits * n;
  const dim3 grid((n + PT - 1) / PT, splits);
  plan_lse_partial_kernel<<<grid, PTHREADS, 0, stream>>>(x, n, y, m, d, g, lb, 1.0 / eps, pm, pl);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  plan_lse_merge_kernel<<<(n + 255) / 256, 256, 0, stream>>>(pm, pl, n, splits, f, la, 1.0 / eps, out);
  return cudaGetLastError();
}

}  // namespace trnopt
