// Shared device/host pieces of the fused Sinkhorn half-step kernels (sm_100a).
//
// The half-step of trnopt (reference src/trnopt/sinkhorn.py:108-119) computes, for every row i of one cloud,
//     lse_i = log sum_j exp( z_ij ),   z_ij = (2 x_i . y_j + gh_j) / eps + log b_j
//     fh_i  = kappa * (|x_i|^2 + eps * off_i - eps * lse_i) - |x_i|^2
// The kernels here keep z in registers (never in memory) in base-2 units, t_ij = z_ij * log2(e), and carry an
// online (max M, sum l) pair per row, sum l = sum_j 2^(t_ij - M).
//
// Work split ("stream-K"): the (row tile, column tile) grid is linearised row-major into U units and CTA k of G
// takes units [k U / G, (k+1) U / G). A CTA's run inside one row tile is a segment; every segment ends with a
// partial (M, l) per row written to the workspace and one arrival on the row tile's counter. The arrival that
// completes a row tile merges its partials and writes the output rows, then resets the counter to zero, so the
// workspace is left ready for the next launch on the same stream.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/trnopt_cuda.h"

namespace trnopt {

constexpr float kLog2e = 1.4426950408889634f;
constexpr double kLn2 = 0.6931471805599453;
// Running-max floor: below every real score (padding scores are about -1.4e9 in base-2 units) and finite, so
// 2^(t - M) never sees inf - inf. Columns past m get bias -inf and contribute exactly 0.
constexpr float kMaxFloor = -1.0e30f;
// Lazy max of the tensor-core epilogue: terms 2^(t - M) are allowed up to 2^kLazyMax before M is raised, so a row
// sum stays below 2^(kLazyMax + 31) for any m < 2^31 (far from FP32 overflow) and rounding stays relative.
constexpr float kLazyMax = 20.0f;
constexpr float kLazyRedo = 100.0f;      // a sum of 32 terms below 2^100 cannot have overflowed FP32
constexpr float kLazyHeadroom = 8.0f;

// Device error word: bit flags set by kernels that give up a bounded wait. Read and cleared by the host API.
enum ErrorBits : int {
  kErrWaitTimeout = 1,   // an mbarrier / pipeline wait ran out of its time limit
  kErrTmemAlloc = 2,     // tensor-memory allocation did not return in time
  kErrBadLaunch = 4,     // a launch-shape invariant did not hold on the device
  kErrPeerTimeout = 8,   // another GPU of the job did not publish its rows within the time limit
};

struct LseProblem {
  const float* xT;     // row side points, transposed: xT[k * ldx + i], k < d, i < rows
  int ldx;
  const float* yT;     // column side points, transposed: yT[k * ldy + j], j < m
  int ldy;
  const float* gh;     // (m,) shifted potential of the column side; nullptr = 0
  const float* log_b;  // (m,) log weights of the column side; nullptr = 0
  const float* xsq;    // (rows,) |x_i|^2 (fh mode only)
  const float* off;    // (rows,) log(target / reference) of the rows; nullptr = 0 (fh mode only)
  int rows, m, d;
  float dot2;          // multiplier of x.y in base-2 units: 2 log2(e) / eps (fh) or log2(e) (lse)
  float gh2;           // multiplier of gh: log2(e) / eps
  float lb2;           // multiplier of log b: log2(e)
  double eps, kappa;   // fh epilogue
  int mode;            // 0: write fh, 1: write lse (natural log)
  float* out;          // (rows,)
  int* error_word;     // device error flags
  const TrnoptSolveState* dyn;   // nullptr, or the solve state whose stage gives eps and kappa (and done: return)
  int side;            // with dyn: 0 = the f half-step (kappa[0]), 1 = the g half-step (kappa[1])
};

// Stream-K bookkeeping, computed on the host per launch.
struct StreamK {
  int nrt, nct;        // row tiles, column tiles
  long long units;     // nrt * nct
  int grid;            // G, <= units
  int slots;           // partial slots per row tile and per producer (>= the most CTAs touching a row tile)
  int parts_per_cta;   // partials one CTA writes per segment (1 for the FFMA kernel, 2 for the tcgen05 kernel)
  int* counters;       // (nrt,) arrival counters, zero between launches
  float2* partials;    // (nrt, slots * parts_per_cta, BM) of (M, l)
  int rotate = 0;      // tcgen05 kernel: sweep each row tile's column tiles in the CTAs' common phase
};

__host__ __device__ inline long long sk_unit_begin(long long k, long long units, long long grid) {
  return (k * units) / grid;
}

// The CTA whose range holds unit u: the largest k with floor(k U / G) <= u, i.e. ceil((u + 1) G / U) - 1.
__host__ __device__ inline int sk_cta_of(long long u, long long units, long long grid) {
  return (int)(((u + 1) * grid + units - 1) / units - 1);
}

// Host: size the partial buffer. A row tile of nct units can be touched by at most ceil(nct G / U) + 1 CTAs.
inline int sk_max_slots(long long units, long long grid, int nct) {
  long long s = (nct * grid + units - 1) / units + 1;
  return (int)s;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Merge of two online (max, sum) pairs in base 2.
__device__ __forceinline__ void lse_merge(float& M, float& l, float M2, float l2) {
  float Mn = fmaxf(M, M2);
  l = l * ex2_approx(M - Mn) + l2 * ex2_approx(M2 - Mn);
  M = Mn;
}

// Finish one row: merge nparts partials (M, l) and apply the kappa / off epilogue (reference src/trnopt/sinkhorn.py:119,
// src/trnopt/nki_sinkhorn.py:212-225). The loads of the first kRegParts partials and of the row's own inputs are
// issued together (one memory round trip for the usual 2-8 partials); the merge order is the partials' order either
// way. The weights 2^(M_k - M) <= 1 come from ex2.approx (relative error ~2^-22, the level of the terms inside each
// partial) and are summed with the partials in double precision, as is the rest of the epilogue. (Double-precision
// exp2 here, inlined at every merge site, measured 4-7 % slower for the whole tensor-core kernel.)
// The (max, sum) of K partials held in registers: every load in flight at once, so one L2 round trip.
template <int K>
__device__ __forceinline__ void parts_lse(const float2* parts, int nparts, int stride, float& M, double& l) {
  float2 v[K];
#pragma unroll
  for (int s = 0; s < K; ++s) v[s] = s < nparts ? __ldcg(&parts[(size_t)s * stride]) : make_float2(kMaxFloor, 0.f);
  M = kMaxFloor;
#pragma unroll
  for (int s = 0; s < K; ++s) M = fmaxf(M, v[s].x);
  l = 0.0;
#pragma unroll
  for (int s = 0; s < K; ++s)
    if (v[s].y > 0.f) l += (double)v[s].y * (double)ex2_approx(v[s].x - M);
}

// More than 8 partials (a row tile spread over more than four CTAs of the tcgen05 kernel: small problems): up to 16
// in one round of loads, the rest by a loop. Out of line, so the merge sites in the hot loops stay small.
struct PartsLse {
  float M;
  double l;
};
static __device__ __noinline__ PartsLse parts_lse_wide(const float2* parts, int nparts, int stride) {
  constexpr int kW = 16;
  PartsLse r;
  parts_lse<kW>(parts, nparts, stride, r.M, r.l);
  if (nparts > kW) {
    float M = r.M;
    for (int s = kW; s < nparts; ++s) M = fmaxf(M, __ldcg(&parts[(size_t)s * stride].x));
    double l = r.l * (double)ex2_approx(r.M - M);
    for (int s = kW; s < nparts; ++s) {
      const float2 w = __ldcg(&parts[(size_t)s * stride]);
      if (w.y > 0.f) l += (double)w.y * (double)ex2_approx(w.x - M);
    }
    r.M = M;
    r.l = l;
  }
  return r;
}

// kWide: more than 8 partials go through parts_lse_wide (one round of loads for up to 16); for a merge that nothing
// overlaps (the end of a CTA's range). Otherwise they are read by two short loops, which keep the merge site small.
template <bool kWide = false>
__device__ inline float finish_row(const LseProblem& p, int row, const float2* parts, int nparts, int stride,
                                   double eps, double kappa) {
  constexpr int kRegParts = 8;
  const float xsq = p.mode == 0 ? __ldg(p.xsq + row) : 0.f;
  const float off = (p.mode == 0 && p.off) ? __ldg(p.off + row) : 0.f;
  float M;
  double l;
  if (kWide && nparts > kRegParts) {
    const PartsLse r = parts_lse_wide(parts, nparts, stride);
    M = r.M;
    l = r.l;
  } else {
    float2 v[kRegParts];
#pragma unroll
    for (int s = 0; s < kRegParts; ++s)
      v[s] = s < nparts ? __ldcg(&parts[(size_t)s * stride]) : make_float2(kMaxFloor, 0.f);
    M = kMaxFloor;
#pragma unroll
    for (int s = 0; s < kRegParts; ++s) M = fmaxf(M, v[s].x);
    for (int s = kRegParts; s < nparts; ++s) M = fmaxf(M, __ldcg(&parts[(size_t)s * stride].x));
    l = 0.0;
#pragma unroll
    for (int s = 0; s < kRegParts; ++s)
      if (v[s].y > 0.f) l += (double)v[s].y * (double)ex2_approx(v[s].x - M);
    for (int s = kRegParts; s < nparts; ++s) {
      const float2 w = __ldcg(&parts[(size_t)s * stride]);
      if (w.y > 0.f) l += (double)w.y * (double)ex2_approx(w.x - M);
    }
  }
  double lse = ((double)M + log2(l)) * kLn2;
  double res;
  if (p.mode == 0) {
    res = kappa * ((double)xsq + eps * (double)off - eps * lse) - (double)xsq;
  } else {
    res = lse;
  }
  p.out[row] = (float)res;
  return (float)res;
}

// Bounded-wait helpers ---------------------------------------------------------------------------------------

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

constexpr unsigned long long kWaitLimitNs = 4000000000ull;   // 4 s: no legitimate wait in these kernels is close

// Publishing a half-step's rows to the other GPUs of a job ------------------------------------------------------
//
// With one process per GPU and the rows of a half-step split over the GPUs, every GPU needs the whole new potential
// before the next half-step. Instead of an all-gather after the kernel, the kernel's epilogue stores each finished
// row into every GPU's copy of the output vector (peer memory over NVLink), and the last CTA to finish raises this
// GPU's flag in every other GPU's flag array to the launch's epoch. A later launch reads its input only after every
// other GPU's flag has reached the epoch it depends on. The flags live in each GPU's own memory; slot q of a GPU's
// array is written only by GPU q.
constexpr int kMaxRanks = 8;

struct Publish {
  int world;                                   // GPUs in the job; 1 = nothing to publish or wait for
  int rank;                                    // this GPU's index in the job
  float* out_peer[kMaxRanks];                  // this launch's output rows as mapped in each GPU's copy
  unsigned long long* flag_peer[kMaxRanks];    // slot `rank` of each GPU's flag array
  const unsigned long long* flags;             // this GPU's flag array (slot q written by GPU q)
  unsigned long long wait_epoch;               // the input is complete once every other slot is >= wait_epoch
  unsigned long long epoch;                    // written to every other GPU when this launch is complete
  int* done;                                   // CTAs of this launch that have finished (zero between launches)
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait (all 32 lanes of a warp) until every other GPU's slot reaches pub.wait_epoch: lane q watches GPU q, so the
// wait lasts as long as the latest GPU, not the sum of the polls. Bounded: false on every lane after kWaitLimitNs,
// with kErrPeerTimeout set in the error word. Loads after it, by any lane, see the peers' rows (__syncwarp).
__device__ inline bool wait_peers(const Publish& pub, int* error_word) {
  const int lane = threadIdx.x & 31;
  const bool watch = lane < pub.world && lane != pub.rank;
  const unsigned long long t0 = globaltimer_ns();
  bool mine = !watch;
  for (;;) {
    if (!mine) mine = ld_acquire_sys(pub.flags + lane) >= pub.wait_epoch;
    if (__all_sync(0xffffffffu, mine)) break;
    if (__any_sync(0xffffffffu, globaltimer_ns() - t0 > kWaitLimitNs)) {   // one decision for the whole warp
      if (lane == 0) atomicOr(error_word, (int)kErrPeerTimeout);
      __syncwarp();
      return false;
    }
    __nanosleep(64);
  }
  __syncwarp();
  return true;
}

// Store one finished row into the other GPUs' copies (the local copy is written by finish_row).
__device__ __forceinline__ void publish_row(const Publish& pub, int row, float v) {
  for (int q = 0; q < pub.world; ++q)
    if (q != pub.rank) pub.out_peer[q][row] = v;
}

// Called by one thread of each CTA after the CTA's last publish_row (every writer has executed
// __threadfence_system(), so its peer stores are complete, and passed a CTA barrier since; a GPU-scope fence
// orders this CTA's arrival after them). The last CTA of the grid raises this GPU's slot to pub.epoch on every
// other GPU (system-scope release) and re-arms the counter.
__device__ inline void publish_done(const Publish& pub) {
  __threadfence();
  if (atomicAdd(pub.done, 1) == (int)gridDim.x - 1) {
    __threadfence_system();
    for (int q = 0; q < pub.world; ++q)
      if (q != pub.rank) st_release_sys(pub.flag_peer[q], pub.epoch);
    atomicExch(pub.done, 0);
  }
}

}  // namespace trnopt
