// Device-side set-up and tear-down of a solve: the per-coordinate statistics of the clouds, the clouds in the
// half-step kernels' layout, and the potentials unshifted into float64 for the download.
//
// The reference builds its device layout on the host (src/trnopt/sinkhorn.py:131-167, _Cloud: padding, squared
// norms in float64 then cast, log weights with PAD_LOG_WEIGHT on padding, the weights, the row offsets) after
// normalising on the host (:268-269), and unshifts on the way out (:375-376). Here one float64 upload per cloud is
// followed by:
//   cloud_stats_kernel     per-coordinate sum, min and max of both clouds (fixed partition and reduction order, so
//                          the result is the same on every run); the host turns them into this package's internal
//                          frame (a translation that puts the joint mean at the origin) and the FP16 split scale
//   prepare_cloud_kernel   one warp per point: the translated coordinates in float64, |x|^2 in float64, the FP16
//                          [hi | lo] row of the tensor-core path (or the FP32 transposed row of the FFMA path), the
//                          float32 vectors, and (column cloud) the initial shifted potential
//   unshift_kernel         f = fh + |x|^2 in float64 into the caller's download buffer
//   take_error_kernel      the device error word into the same buffer (and cleared), so one copy brings back
//                          potentials and error flags together
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "../../include/trnopt_cuda.h"
#include "kernels.h"

namespace trnopt {
namespace {

constexpr int kStatsThreads = 256;
constexpr int kMaxD = 128;

int stats_blocks(int device) {
  static std::atomic<int> sms[kMaxDevices];
  if (device < 0 || device >= kMaxDevices) device = 0;
  int s = sms[device].load();
  if (s == 0) {
    cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, device);
    if (s <= 0) s = 148;
    sms[device].store(s);
  }
  return 2 * s;
}

// Threads of a block: coordinate k = t % dpad (dpad = d rounded up to a power of two), row lane t / dpad.
__device__ __forceinline__ int pow2_at_least(int d) {
  int p = 1;
  while (p < d) p <<= 1;
  return p;
}

// grid (B, 2): block b of cloud c reduces rows [b R, (b + 1) R) of that cloud into partial[c][b][3][d]; the last block
// of a cloud to finish reduces the B partials in block order into stats[c][3][d] and re-arms the cloud's counter.
__global__ void __launch_bounds__(kStatsThreads) cloud_stats_kernel(const double* __restrict__ x, int n,
                                                                    const double* __restrict__ y, int m, int d,
                                                                    double* __restrict__ partial,
                                                                    int* __restrict__ counters,
                                                                    double* __restrict__ stats) {
  __shared__ double s_sum[kStatsThreads], s_min[kStatsThreads], s_max[kStatsThreads];
  __shared__ int s_last;
  const int c = blockIdx.y;
  const double* __restrict__ p = c == 0 ? x : y;
  const int count = c == 0 ? n : m;
  const int B = gridDim.x, b = blockIdx.x;
  const int dpad = pow2_at_least(d), lanes = kStatsThreads / dpad;
  const int k = threadIdx.x % dpad, lane = threadIdx.x / dpad;
  const long long R = ((long long)count + B - 1) / B;
  const long long r0 = (long long)b * R, r1 = min((long long)count, r0 + R);
  double sum = 0.0, mn = INFINITY, mx = -INFINITY;
  if (k < d) {
#pragma unroll 4
    for (long long r = r0 + lane; r < r1; r += lanes) {
      const double v = __ldg(p + r * d + k);
      sum += v;
      mn = fmin(mn, v);
      mx = fmax(mx, v);
    }
  }
  s_sum[threadIdx.x] = sum;
  s_min[threadIdx.x] = mn;
  s_max[threadIdx.x] = mx;
  __syncthreads();
  double* part = partial + ((size_t)c * B + b) * 3 * d;
  if (threadIdx.x < d) {
    double a = 0.0, lo = INFINITY, hi = -INFINITY;
    for (int l = 0; l < lanes; ++l) {                       // lanes in order
      const int t = l * dpad + threadIdx.x;
      a += s_sum[t];
      lo = fmin(lo, s_min[t]);
      hi = fmax(hi, s_max[t]);
    }
    part[threadIdx.x] = a;
    part[d + threadIdx.x] = lo;
    part[2 * d + threadIdx.x] = hi;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[c], 1) == B - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x < d) {
    double a = 0.0, lo = INFINITY, hi = -INFINITY;
    const double* base = partial + (size_t)c * B * 3 * d;
    for (int q = 0; q < B; ++q) {                           // blocks in order
      const double* pq = base + (size_t)q * 3 * d;
      a += __ldcg(pq + threadIdx.x);
      lo = fmin(lo, __ldcg(pq + d + threadIdx.x));
      hi = fmax(hi, __ldcg(pq + 2 * d + threadIdx.x));
    }
    double* st = stats + (size_t)c * 3 * d;
    st[threadIdx.x] = a;
    st[d + threadIdx.x] = lo;
    st[2 * d + threadIdx.x] = hi;
  }
  if (threadIdx.x == 0) counters[c] = 0;
}

struct PrepArgs {
  const double* pts;     // (n, d) row-major, float64
  int n, d, npad, dk, kp;
  double r;              // coordinates become (p - center) / r - shift
  float scale;           // 2^scale_exp for the FP16 split
  const double* log_w;   // (n,) or nullptr: every point has log weight log_w_uniform
  double log_w_uniform;
  const double* off;     // (n,) or nullptr (0)
  __half* packed;        // (npad, kp) or nullptr
  float* xT;             // (d, npad) or nullptr
  float* vec;            // (4, npad): |x|^2, log w, w, off  (float32)
  double* sq64;          // (npad,) |x|^2 in float64
  float* gh0;            // (npad,) or nullptr: |x_s|^2 - |x|^2 (the reference's initial g = |y|^2 in its frame)
  double center[kMaxD];
  double shift[kMaxD];
};

constexpr int kPrepWarps = 8;
constexpr double kPadLogWeight = -1e9;

__global__ void __launch_bounds__(kPrepWarps * 32) prepare_cloud_kernel(const PrepArgs a) {
  const int lane = threadIdx.x & 31;
  const long long i = (long long)blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
  if (i >= a.npad) return;
  const bool real = i < a.n;
  constexpr int J = kMaxD / 32;
  double xi[J];
  double ss = 0.0, si = 0.0;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int k = lane + 32 * j;
    xi[j] = 0.0;
    if (real && k < a.d) {
      const double xs = (__ldg(a.pts + i * a.d + k) - a.center[k]) / a.r;
      const double v = xs - a.shift[k];
      xi[j] = v;
      ss = fma(xs, xs, ss);
      si = fma(v, v, si);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    si += __shfl_xor_sync(0xffffffffu, si, o);
  }
  if (a.packed) {
    __half* row = a.packed + i * a.kp;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int k = lane + 32 * j;
      if (k < a.dk) {
        __half hi = __float2half_rn(0.f), lo = __float2half_rn(0.f);
        if (k < a.d) {
          const float v = (float)xi[j] * a.scale;              // exact: the scale is a power of two
          hi = __float2half_rn(v);
          lo = __float2half_rn(v - __half2float(hi));
        }
        row[k] = hi;
        row[a.dk + k] = lo;
      }
    }
    for (int e = 2 * a.dk + lane; e < a.kp; e += 32) row[e] = __float2half_rn(0.f);
  }
  if (a.xT) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int k = lane + 32 * j;
      if (k < a.d) a.xT[(size_t)k * a.npad + i] = (float)xi[j];
    }
  }
  if (lane == 0) {
    const double lw = real ? (a.log_w ? __ldg(a.log_w + i) : a.log_w_uniform) : kPadLogWeight;
    const double of = (real && a.off) ? __ldg(a.off + i) : 0.0;
    a.vec[i] = (float)si;
    a.vec[a.npad + i] = (float)lw;
    a.vec[2 * (size_t)a.npad + i] = (float)exp(lw);
    a.vec[3 * (size_t)a.npad + i] = (float)of;
    a.sq64[i] = si;
    if (a.gh0) a.gh0[i] = (float)(ss - si);
  }
}

__global__ void unshift_kernel(const float* __restrict__ h, const double* __restrict__ sq, int n,
                               const double* __restrict__ gauge, double sign, double* __restrict__ out) {
  const double c = gauge ? sign * gauge[0] : 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = ((double)h[i] + sq[i]) + c;
}

__global__ void take_error_kernel(int* word, double* out) { out[0] = (double)atomicExch(word, 0); }

bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

}  // namespace
}  // namespace trnopt

using namespace trnopt;

extern "C" {

size_t trnopt_cloud_stats_scratch_bytes(int d) {
  if (d < 1 || d > kMaxD) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  return 256 + (size_t)2 * stats_blocks(dev) * 3 * d * sizeof(double);
}

int trnopt_cloud_stats(const double* x, int n, const double* y, int m, int d, double* stats, void* scratch,
                       size_t scratch_bytes, void* stream) {
  if (!x || !y || !stats || !scratch || n < 1 || m < 1 || d < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (d > kMaxD) return TRNOPT_ERR_UNSUPPORTED;
  if (scratch_bytes < trnopt_cloud_stats_scratch_bytes(d)) return TRNOPT_ERR_WORKSPACE;
  if (!aligned8(x) || !aligned8(y) || !aligned8(stats) || (reinterpret_cast<uintptr_t>(scratch) & 255u))
    return TRNOPT_ERR_ALIGNMENT;
  int dev = 0;
  cudaGetDevice(&dev);
  const int B = stats_blocks(dev);
  int* counters = static_cast<int*>(scratch);
  double* partial = reinterpret_cast<double*>(static_cast<char*>(scratch) + 256);
  cloud_stats_kernel<<<dim3(B, 2), kStatsThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, n, y, m, d, partial,
                                                                                               counters, stats);
  return cudaGetLastError() == cudaSuccess ? TRNOPT_OK : TRNOPT_ERR_CUDA;
}

int trnopt_prepare_cloud(const double* pts, int n, int d, int npad, const double* center, double r,
                         const double* shift, int scale_exp, const double* log_w, double log_w_uniform,
                         const double* off, void* packed, float* xT, float* vec, double* sq64, float* gh0,
                         void* stream) {
  if (!pts || !center || !shift || !vec || !sq64 || n < 1 || d < 1 || npad < n) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!(r > 0.0) || !isfinite(r) || !isfinite(log_w_uniform) || scale_exp < -100 || scale_exp > 100)
    return TRNOPT_ERR_INVALID_ARGUMENT;
  if (d > kMaxD) return TRNOPT_ERR_UNSUPPORTED;
  if (packed && !tc_supported_d(d)) return TRNOPT_ERR_UNSUPPORTED;
  if (!aligned8(pts) || !aligned8(sq64) || (log_w && !aligned8(log_w)) || (off && !aligned8(off)) ||
      (reinterpret_cast<uintptr_t>(vec) & 3u) || (packed && (reinterpret_cast<uintptr_t>(packed) & 127u)))
    return TRNOPT_ERR_ALIGNMENT;
  PrepArgs a{};
  a.pts = pts;
  a.n = n;
  a.d = d;
  a.npad = npad;
  a.dk = packed ? tc_supported_d(d) : 0;
  a.kp = packed ? tc_kp(d) : 0;
  a.r = r;
  a.scale = ldexpf(1.0f, scale_exp);
  a.log_w = log_w;
  a.log_w_uniform = log_w_uniform;
  a.off = off;
  a.packed = static_cast<__half*>(packed);
  a.xT = xT;
  a.vec = vec;
  a.sq64 = sq64;
  a.gh0 = gh0;
  for (int k = 0; k < d; ++k) {
    a.center[k] = center[k];
    a.shift[k] = shift[k];
  }
  const unsigned blocks = (unsigned)((npad + kPrepWarps - 1) / kPrepWarps);
  prepare_cloud_kernel<<<blocks, kPrepWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? TRNOPT_OK : TRNOPT_ERR_CUDA;
}

int trnopt_unshift(const float* h, const double* sq, int n, const double* gauge, int sign, double* out,
                   void* stream) {
  if (!h || !sq || !out || n < 1 || (sign != 1 && sign != -1)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned8(sq) || !aligned8(out) || (gauge && !aligned8(gauge))) return TRNOPT_ERR_ALIGNMENT;
  const int blocks = (n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184;
  unshift_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(h, sq, n, gauge, (double)sign, out);
  return cudaGetLastError() == cudaSuccess ? TRNOPT_OK : TRNOPT_ERR_CUDA;
}

int trnopt_take_error_flags(double* out, void* stream) {
  if (!out) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned8(out)) return TRNOPT_ERR_ALIGNMENT;
  int* word = device_error_word();
  if (!word) return TRNOPT_ERR_CUDA;
  take_error_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(word, out);
  return cudaGetLastError() == cudaSuccess ? TRNOPT_OK : TRNOPT_ERR_CUDA;
}

}  // extern "C"
