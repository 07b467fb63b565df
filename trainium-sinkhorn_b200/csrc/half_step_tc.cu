// Fused Sinkhorn half-step on the 5th-generation tensor cores (tcgen05, sm_100a), split precision.
//
// The contraction x_i . y_j runs as three FP16 tensor-core products with FP32 accumulation in tensor memory,
//     x . y ~= 2^-(sx+sy) * ( xh . yh + xh . yl + xl . yh ),   x 2^sx = xh + xl,  y 2^sy = yh + yl  (FP16 pairs)
// where the power-of-two scales put each cloud's largest coordinate in (2^13, 2^14] (so the low halves of typical
// coordinates are normal FP16 numbers) and the low halves carry the next 11 bits, so the products keep about
// 22 significant bits (FP32-level; a plain FP16 or TF32 product
// keeps 11, which moves plans by percents -- the reference's README reports 2-3.5% for TF32). The points do not
// change during a solve, so each cloud is split once (tc_pack) into rows of [hi (dk) | lo (dk)] FP16 values.
//
// Per CTA (one per SM, persistent over a stream-K range of (128-row tile, 256-column tile) units):
//   warp 8      TMA producer: row tiles (A, two buffers) and column tiles (B, a ring of stages) into 128B-swizzled
//               shared memory.
//   warp 10     the tile's column bias b_j = (gh_j / eps + log b_j) log2(e), written as b_j / dot2 in three BF16
//               parts into one of two MMA operand slots (K 0..2 of row j).
//   warp 9      allocates 512 TMEM columns and issues the MMAs (M 128, N 256, K 16; 3 dk / 16 FP16 MMAs per tile,
//               then one BF16 MMA of a constant [1, 1, 1, 0 ...] tile with the bias slot, which adds b_j / dot2)
//               into one of two 128 x 256 FP32 accumulators, committing to mbarriers.
//   warps 0-7   two epilogue warpgroups, each on half the columns of every tile: a thread owns one row, reads its
//               128 scores of a tile from TMEM 64 at a time, scales them by dot2 and folds them into an online
//               (max, sum) in base 2 (MUFU ex2, lazy max; see lse_tile128). The accumulator is released as soon
//               as the tile's TMEM reads are done, before the last exps. At the end of a segment each warpgroup
//               writes its partial; the last arrival for a row tile merges all partials and writes fh (common.cuh).
// Every mbarrier wait is bounded (common.cuh kWaitLimitNs); a timeout sets the device error word and the CTA
// unwinds (waits for its own copies and MMAs, frees TMEM) instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace trnopt {

constexpr int TC_BM = 128;          // rows per tile (MMA M, TMEM lanes)
constexpr int TC_BN = 256;          // columns per tile (MMA N)
constexpr int TC_NACC = 2;          // TMEM accumulators of TC_BN columns (512 columns in all)
constexpr int TC_THREADS = 352;     // 8 epilogue warps + TMA producer + MMA + bias
constexpr int TC_NBB = 2;           // column-bias operand slots (one per tile in flight between bias warp and MMA)
constexpr int kTcPolyExps = 8;     // of every 64 exps of the fold, how many run on the FMA pipe
constexpr int TC_PRODUCER_WARP = 8;
constexpr int TC_MMA_WARP = 9;
constexpr int TC_BIAS_WARP = 10;

// ------------------------------------------------------------------------------------------------------------
// PTX wrappers
// ------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// A waiting thread sleeps in try_wait until the phase completes or kWaitHintNs pass. The producer, bias and MMA
// warps spend most of their time waiting, on the same sub-partitions as the epilogue warps: every poll is an issue
// slot taken from the epilogue, so the polls are kept rare (the wake-up on completion does not wait for the hint).
constexpr uint32_t kWaitHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kWaitHintNs)
      : "memory");
  return ok != 0;
}

// Bounded wait: spin on try_wait; every 256 polls look at the clock and (unless draining) at the CTA's abort flag.
// Draining waits (for our own copies and MMAs before exit) ignore the abort flag but keep the time limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* error_word,
                                          bool draining = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (!draining && *abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicOr(error_word, (int)kErrWaitTimeout);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define TRNOPT_TMEM_LD64(taddr, v) \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];" \
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63]) \
               : "r"(taddr) : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzle layout: rows of 128 bytes,
// 8-row atoms of 1024 bytes stacked along M/N (stride byte offset 1024), start address in 16-byte units.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)1u << 16;                           // leading byte offset (unused with swizzling; 16 B)
  d |= (uint64_t)(1024u >> 4) << 32;                 // stride byte offset: 1024 B between 8-row groups
  d |= (uint64_t)1u << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                           // layout: 128-byte swizzle
  return d;
}

// Packed FP32 pair arithmetic (sm_100): two lanes of work per instruction on the FMA pipe.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// One block of 64 values of a row relative to `shift` (the row's running max M): u_j = acc_j * dot2 - shift, one
// packed FMA per two values (the column bias is already in the accumulator), their max, and the values in a[].
template <int N>
__device__ __forceinline__ void block_terms(uint32_t (&v)[N], uint64_t d2, float shift, float (&a)[N], float& cmax) {
  const uint64_t nm = pk2(-shift, -shift);
#pragma unroll
  for (int q = 0; q < N / 2; ++q) {
    const uint64_t u = ffma2(pk2(__uint_as_float(v[2 * q]), __uint_as_float(v[2 * q + 1])), d2, nm);
    upk2(u, a[2 * q], a[2 * q + 1]);
  }
  float c[4];                                                 // chain k reduces every fourth group of 8
#pragma unroll
  for (int k = 0; k < 4; ++k) c[k] = kMaxFloor;
#pragma unroll
  for (int g = 0; g < N / 8; ++g) {
    const int b = 8 * g, k = g & 3;
    c[k] = fmax3(c[k], a[b], a[b + 1]);
    c[k] = fmax3(c[k], a[b + 2], a[b + 3]);
    c[k] = fmax3(c[k], a[b + 4], a[b + 5]);
    c[k] = fmax3(c[k], a[b + 6], a[b + 7]);
  }
  cmax = fmaxf(fmaxf(c[0], c[1]), fmaxf(c[2], c[3]));
}

// 2^x on the FMA pipe, to take a share of the exps off MUFU (16 results / clock / SM). Range reduction by the
// round-to-integer add (x + 1.5 * 2^23 keeps round(x) in the low mantissa bits), 2^f on [-1/2, 1/2] by a degree-5
// polynomial fitted for this library (relative minimax, Lawson-iterated least squares; fit error 7.5e-8), and the
// integer part added to the exponent field. Max relative error 2.1e-7 over [-125, 100] (ex2.approx: ~2^-22).
// Inputs below -125 are clamped (their terms are < 2^-125, nothing next to a row's largest term of >= 2^-8).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float y = x + 12582912.0f;
  const float f = x - (y - 12582912.0f);
  float p = 0x1.5c08dcp-10f;
  p = fmaf(p, f, 0x1.3d0c54p-7f);
  p = fmaf(p, f, 0x1.c6b6e6p-5f);
  p = fmaf(p, f, 0x1.ebf918p-3f);
  p = fmaf(p, f, 0x1.62e428p-1f);
  p = fmaf(p, f, 0x1.000002p+0f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(y) << 23));
}

// ex2_poly of a pair with packed FP32 operations: per lane the same IEEE operations in the same order (x - r as
// fma(r, -1, x)), so the same results as two ex2_poly calls, in about half the instructions.
__device__ __forceinline__ uint64_t ex2_poly2(float x0, float x1) {
  const uint64_t x = pk2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t y = fadd2(x, pk2(12582912.0f, 12582912.0f));
  const uint64_t f = ffma2(fadd2(y, pk2(-12582912.0f, -12582912.0f)), pk2(-1.0f, -1.0f), x);
  uint64_t p = ffma2(pk2(0x1.5c08dcp-10f, 0x1.5c08dcp-10f), f, pk2(0x1.3d0c54p-7f, 0x1.3d0c54p-7f));
  p = ffma2(p, f, pk2(0x1.c6b6e6p-5f, 0x1.c6b6e6p-5f));
  p = ffma2(p, f, pk2(0x1.ebf918p-3f, 0x1.ebf918p-3f));
  p = ffma2(p, f, pk2(0x1.62e428p-1f, 0x1.62e428p-1f));
  p = ffma2(p, f, pk2(0x1.000002p+0f, 0x1.000002p+0f));
  float p0, p1, y0, y1;
  upk2(p, p0, p1);
  upk2(y, y0, y1);
  return pk2(__uint_as_float(__float_as_uint(p0) + (__float_as_uint(y0) << 23)),
             __uint_as_float(__float_as_uint(p1) + (__float_as_uint(y1) << 23)));
}

// 2^x of a pair: on the FMA pipe (ex2_poly2) when `poly`, else on MUFU (ex2.approx). (`poly` is a constant once
// the callers' loops are unrolled.)
__device__ __forceinline__ uint64_t ex2_pair(bool poly, float x, float y) {
  return poly ? ex2_poly2(x, y) : pk2(ex2_approx(x), ex2_approx(y));
}

// sum_j 2^(a_j - off), four independent packed partial sums. kPoly of every 64 values (spread evenly over the value
// pairs) take the FMA-pipe polynomial, the rest MUFU: MUFU does 16 exps per clock per SM, and the fold has issue
// slots and FMA-pipe cycles to spare beside it.
template <int N, int kPoly = 0>
__device__ __forceinline__ float exp_sum(const float (&a)[N], float off) {
  uint64_t s0 = 0ull, s1 = 0ull, s2 = 0ull, s3 = 0ull;
  constexpr int kPolyPairs = kPoly / 2;
#define TRNOPT_POLY_PAIR(pair) (kPolyPairs > 0 && ((pair) * kPolyPairs) % (N / 2) < kPolyPairs)
#pragma unroll
  for (int j = 0; j < N; j += 8) {
    s0 = fadd2(s0, ex2_pair(TRNOPT_POLY_PAIR(j / 2), a[j] - off, a[j + 1] - off));
    s1 = fadd2(s1, ex2_pair(TRNOPT_POLY_PAIR(j / 2 + 1), a[j + 2] - off, a[j + 3] - off));
    s2 = fadd2(s2, ex2_pair(TRNOPT_POLY_PAIR(j / 2 + 2), a[j + 4] - off, a[j + 5] - off));
    s3 = fadd2(s3, ex2_pair(TRNOPT_POLY_PAIR(j / 2 + 3), a[j + 6] - off, a[j + 7] - off));
  }
#undef TRNOPT_POLY_PAIR
  s0 = fadd2(s0, s1);
  s2 = fadd2(s2, s3);
  s0 = fadd2(s0, s2);
  float x0, x1;
  upk2(s0, x0, x1);
  return x0 + x1;
}

// Redo of one 64-value block in absolute terms from the raw accumulators re-read from TMEM; returns the new
// (M, L). The relative values lose their low bits when M is far below the block (e.g. M set by columns of
// PAD_LOG_WEIGHT, -1e9). Warp-uniform entry (tcgen05.ld is .sync.aligned); lanes without `redo` get (M, L) back
// unchanged. Rarely taken, so it is a call rather than inlined: its two copies would otherwise sit in the hot loop's
// code (inlined, the kernel measured ~3 % slower).
static __device__ __noinline__ float2 block_redo(uint32_t taddr, float dot2, bool redo, float M, float L) {
  constexpr int N = 64;
  uint32_t raw[N];
  TRNOPT_TMEM_LD64(taddr, raw);
  tmem_wait_ld();
  if (!redo) return make_float2(M, L);
  float a[N];
  float tmax = kMaxFloor;
#pragma unroll
  for (int q = 0; q < N / 4; ++q) {
    a[4 * q + 0] = __uint_as_float(raw[4 * q + 0]) * dot2;
    a[4 * q + 1] = __uint_as_float(raw[4 * q + 1]) * dot2;
    a[4 * q + 2] = __uint_as_float(raw[4 * q + 2]) * dot2;
    a[4 * q + 3] = __uint_as_float(raw[4 * q + 3]) * dot2;
    tmax = fmaxf(tmax, fmaxf(fmaxf(a[4 * q], a[4 * q + 1]), fmaxf(a[4 * q + 2], a[4 * q + 3])));
  }
  const float Mn = tmax + kLazyHeadroom;
  return make_float2(Mn, L * ex2_approx(M - Mn) + exp_sum(a, Mn));
}

// Lazy-max update of (M, L) with a block whose values a[] are relative to M: the exps use the
// max known before the block, so no exp waits for the block's max (reduced alongside). Terms may exceed 1 by up
// to 2^kLazyMax; a block whose max is higher rescales its sum (no new exps) while no term can have overflowed
// (max <= M + kLazyRedo); returns true when the block must be redone in absolute terms instead.
template <int N>
__device__ __forceinline__ bool block_fold(const float (&a)[N], float cmax, float& M, float& L) {
  const float sum = exp_sum<N, kTcPolyExps>(a, 0.f);
  if (cmax <= kLazyMax) {
    L += sum;
  } else if (cmax <= kLazyRedo) {
    const float off = cmax + kLazyHeadroom;
    L = (L + sum) * ex2_approx(-off);
    M += off;
  } else {
    return true;
  }
  return false;
}

// M for a row's first block (M still at the floor): the block's largest raw value * dot2 + kLazyHeadroom, so the
// block's terms are then formed against it with one rounding like every other block's; the floor again for a block
// of columns past m only (all -inf).
__device__ __forceinline__ float block_start_ref(const uint32_t (&v)[64], float dot2) {
  float c[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int q = 0; q < 32; ++q) c[q & 3] = fmax3(c[q & 3], __uint_as_float(v[2 * q]), __uint_as_float(v[2 * q + 1]));
  return fmaxf(fmaf(fmaxf(fmaxf(c[0], c[1]), fmaxf(c[2], c[3])), dot2, kLazyHeadroom), kMaxFloor);
}

// Fold one row's 128 accumulator values of a tile (TMEM address taddr, 32x32b lanes: this thread's row) into the
// row's running base-2 (M, L):   t_j = acc_j * dot2 (the accumulator holds x.y plus the column bias / dot2),
// L = sum_j 2^(t_j - M). Two blocks of 64 values (u_j = t_j - M from one packed FMA, acc * dot2 - M); a block that
// finds M at the floor (the segment's first) sets M from its own max first. Block 1 is loaded from TMEM while block
// 0's exps run; once block 1 is loaded and its max (and any redo re-read) is done, every TMEM read of the tile is over
// and the accumulator is released (tcgen05 fence, then an arrival on `acc_empty`) before block 1's exps, so the MMAs
// two tiles ahead overlap them. Must be called by all 32 lanes of the warp.
__device__ __forceinline__ void lse_tile128(uint32_t taddr, float dot2, float& M, float& L, uint64_t* acc_empty) {
  constexpr int N = 64;
  const uint64_t d2 = pk2(dot2, dot2);
  uint32_t v[N];
  float a[N];
  float cmax;
  TRNOPT_TMEM_LD64(taddr, v);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < N; ++j) asm volatile("" : "+r"(v[j]));
  // block 0
  if (M == kMaxFloor) M = block_start_ref(v, dot2);
  block_terms(v, d2, M, a, cmax);
  TRNOPT_TMEM_LD64(taddr + (uint32_t)N, v);                   // block 1 into the now-free registers
  bool redo = block_fold(a, cmax, M, L);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < N; ++j) asm volatile("" : "+r"(v[j]));
  if (__any_sync(0xffffffffu, redo)) {
    const float2 r = block_redo(taddr, dot2, redo, M, L);
    M = r.x;
    L = r.y;
  }
  // block 1: terms and max, then its redo re-read if any, then release the accumulator, then the exps
  if (M == kMaxFloor) M = block_start_ref(v, dot2);
  block_terms(v, d2, M, a, cmax);
  redo = cmax > kLazyRedo;
  if (__any_sync(0xffffffffu, redo)) {
    // Rare: lanes without a redo fold block 1 first (a[] is then free), then the warp re-reads it for the others,
    // then releases.
    if (!redo) block_fold(a, cmax, M, L);
    const float2 r = block_redo(taddr + (uint32_t)N, dot2, redo, M, L);
    M = r.x;
    L = r.y;
    tmem_fence_before();
    mbar_arrive(acc_empty);
  } else {
    tmem_fence_before();
    mbar_arrive(acc_empty);
    block_fold(a, cmax, M, L);
  }
}

// Instruction descriptors, kind::f16: D F32, A and B FP16 (kIdesc) or both BF16 (kIdescBf16), K-major,
// N = TC_BN, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                            ((uint32_t)(TC_BM >> 4) << 24);
constexpr uint32_t kIdescBf16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                                ((uint32_t)(TC_BM >> 4) << 24);

// Shared-memory descriptor of a K-major operand without swizzling: 8-row x 16-byte core matrices, `lbo` bytes
// between the two core matrices of a K = 16 (BF16) slice, `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;                           // descriptor version (sm_100); layout 0: no swizzle
  return d;
}

// The column bias enters the accumulator through one more MMA per tile, K = 16 in BF16: A is a constant tile whose
// rows are [1, 1, 1, 0, ...], B holds for each column j the bias_j / dot2 split into three BF16 parts
// (8 + 8 + 8 significant bits, FP32-level), so acc_ij = x_i.y_j (scaled) + bias_j / dot2 and the epilogue needs no
// per-column term. Plain layout: core matrix (row group g, K half h) at g * 256 + h * 128, row r of the group at
// r * 16, element k of the half at 2 k.
constexpr uint32_t kBiasLbo = 128, kBiasSbo = 256;
constexpr int kBiasABytes = TC_BM * 32;      // 128 rows x 16 BF16
constexpr int kBiasBBytes = TC_BN * 32;      // 256 rows x 16 BF16

__device__ __forceinline__ uint32_t bias_row_offset(int row) { return (uint32_t)((row >> 3) * 256 + (row & 7) * 16); }

// x -> three BF16 parts whose sum is x to FP32 precision; -inf (a column past m) -> (-inf, 0, 0).
__device__ __forceinline__ uint2 bias_split(float x) {
  const __nv_bfloat16 h1 = __float2bfloat16_rn(x);
  if (!(x > -INFINITY)) return make_uint2((uint32_t)__bfloat16_as_ushort(h1), 0u);
  const float r1 = x - __bfloat162float(h1);
  const __nv_bfloat16 h2 = __float2bfloat16_rn(r1);
  const __nv_bfloat16 h3 = __float2bfloat16_rn(r1 - __bfloat162float(h2));
  return make_uint2((uint32_t)__bfloat16_as_ushort(h1) | ((uint32_t)__bfloat16_as_ushort(h2) << 16),
                    (uint32_t)__bfloat16_as_ushort(h3));
}

// Column order within a row tile, for column clouds larger than L2 holds comfortably (StreamK::rotate, set by
// tc_plan). Row tile r visits its column tiles starting at tile (nct - p) mod nct, where p is the column phase (unit
// index mod nct) at which the row's owner -- the CTA holding its last unit -- begins its range. Every CTA then
// sweeps the column tiles in step with the others (its tile at local step t is t mod nct, up to its last row), so
// the column tiles in use at one moment are a narrow window of the column cloud instead of all of it: at 262,144
// columns (a 67 MB cloud) the DRAM reads of a launch drop from 6.7 GB (~100 sweeps' worth) to under 1 GB. Any rotation
// covers each column tile once; this one is the same for every CTA that asks, since all of them ask the owner. A
// CTA needs two values: rows that end inside its range are its own, and only its last row can end in a later
// CTA's range. Computed once per CTA by a whole warp: lane i takes the range start of CTA blockIdx.x + i and its
// phase, so the owner is found by a ballot and the start-up path stays two 64-bit divisions deep (the per-tile
// path has none). Without rotation the order is the natural one.
struct TcColumnOrder {
  int phase;              // u_begin mod nct
  int rot_own, rot_last;  // column tile = (u mod nct + rot) mod nct
  __device__ __forceinline__ int of_row(long long row_end, long long u_end) const {
    return row_end <= u_end ? rot_own : rot_last;
  }
};
template <bool kRotate>
__device__ __forceinline__ TcColumnOrder tc_column_order(const StreamK& sk, long long u_begin, int lane) {
  TcColumnOrder o;
  if (!kRotate) {
    o.phase = (int)(u_begin % sk.nct);
    o.rot_own = o.rot_last = 0;
    return o;
  }
  const long long k = (long long)blockIdx.x + lane;
  const long long b = k < sk.grid ? sk_unit_begin(k, sk.units, sk.grid) : sk.units;   // nondecreasing in the lane
  const int ph = (int)(b % sk.nct);
  o.phase = __shfl_sync(0xffffffffu, ph, 0);
  const int ph_end = __shfl_sync(0xffffffffu, ph, 1);   // u_end mod nct (0 when u_end is the last unit + 1)
  const long long u_end = __shfl_sync(0xffffffffu, b, 1);
  o.rot_own = o.phase == 0 ? 0 : sk.nct - o.phase;
  o.rot_last = o.rot_own;
  if (ph_end != 0) {   // the last row runs past u_end: its owner is the CTA whose range holds its last unit
    const long long last = u_end - ph_end + sk.nct - 1;
    const unsigned below = __ballot_sync(0xffffffffu, b <= last);   // lanes 0 .. owner (lane 0 always)
    int p;
    if (below != 0xffffffffu) {
      p = __shfl_sync(0xffffffffu, ph, 31 - __clz(below));
    } else {   // a row tile over more than 31 CTAs (tiny problems): directly
      p = (int)(sk_unit_begin(sk_cta_of(last, sk.units, sk.grid), sk.units, sk.grid) % sk.nct);
    }
    o.rot_last = p == 0 ? 0 : sk.nct - p;
  }
  return o;
}

// ------------------------------------------------------------------------------------------------------------
// The kernel
// ------------------------------------------------------------------------------------------------------------

template <int NKB>
struct TcCfg {
  static constexpr int A_BYTES = NKB * TC_BM * 128;      // one row tile: NKB K-blocks of 128 rows x 128 B
  static constexpr int B_BYTES = NKB * TC_BN * 128;      // one column tile
  static constexpr int NS = NKB == 1 ? 4 : 2;            // column-tile stages
  static constexpr int OFF_B = 2 * A_BYTES;
  static constexpr int OFF_BIAS_A = OFF_B + NS * B_BYTES;                 // constant BF16 tile [1, 1, 1, 0 ...]
  static constexpr int OFF_BIAS_B = OFF_BIAS_A + kBiasABytes;             // TC_NBB column-bias operand slots
  static constexpr int OFF_BAR = OFF_BIAS_B + TC_NBB * kBiasBBytes;
  // barriers: full[NS], empty[NS], a_full[2], a_empty[2], acc_full[NACC], acc_empty[NACC], bias_full[NBB],
  // bias_empty[NBB], drain[1]
  static constexpr int NBAR = 2 * NS + 4 + 2 * TC_NACC + 2 * TC_NBB + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 64 + 1024;     // + alignment slack for the 1024-byte aligned base
};

struct TcArgs {
  LseProblem p;
  StreamK sk;
  int dk;            // elements of each half (hi, lo) per packed row; multiple of 16
  float dot2_scale;  // 2^-(sx + sy): p.dot2 is already scaled; a solve state's dot2 is scaled by this in the kernel
  int mirror;        // 1 when the row cloud lies above the column cloud in memory: correction passes swapped
  Publish pub;       // world > 1: wait for the other GPUs' rows of gh, publish this GPU's rows of the output
};

template <int NKB, bool kRotate>
__global__ void __launch_bounds__(TC_THREADS, 1)
    half_step_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const TcArgs args) {
  using C = TcCfg<NKB>;
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  const LseProblem& p = args.p;
  const StreamK& sk = args.sk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The half-step's scalars: from the arguments, or (a run decided on the device) from the solve state's current
  // stage, read before anything else; a state that is done leaves nothing to do. A launch that reads a state is
  // ordered after the check that last wrote it (launched without programmatic overlap, or within a run in which
  // no check runs).
  float dot2_e = p.dot2, gh2_e = p.gh2;
  double eps_e = p.eps, kappa_e = p.kappa;
  if (p.dyn != nullptr) {
    const TrnoptSolveState* st = p.dyn;
    if (st->done) return;
    dot2_e = st->dot2 * args.dot2_scale;
    gh2_e = st->gh2;
    eps_e = (double)st->eps;
    kappa_e = (double)st->kappa[p.side];
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full_b = bars;
  uint64_t* empty_b = bars + C::NS;
  uint64_t* a_full = bars + 2 * C::NS;
  uint64_t* a_empty = a_full + 2;
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + TC_NACC;
  uint64_t* bias_full = acc_empty + TC_NACC;
  uint64_t* bias_empty = bias_full + TC_NBB;
  uint64_t* drain = bias_empty + TC_NBB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
  int* s_last = reinterpret_cast<int*>(smem + C::OFF_MISC + 16);     // [2], one per epilogue warpgroup
  int* s_pend = reinterpret_cast<int*>(smem + C::OFF_MISC + 24);     // [2][2]: pending row tile, its arrivals

  if (blockDim.x != TC_THREADS) {
    if (threadIdx.x == 0) atomicOr(p.error_word, (int)kErrBadLaunch);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) { mbar_init(&full_b[s], 1); mbar_init(&empty_b[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&a_full[b], 1); mbar_init(&a_empty[b], 1); }
    for (int b = 0; b < TC_NACC; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 256); }
    for (int s = 0; s < TC_NBB; ++s) { mbar_init(&bias_full[s], 32); mbar_init(&bias_empty[s], 1); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  {
    // Bias operands: A rows [1, 1, 1, 0 ... 0] (BF16 1.0 = 0x3F80), B slots zero (the bias warp fills K 0..2 of
    // each row per tile; K 3..15 must stay finite). Written through the generic proxy, read by the tensor core.
    uint4* ba = reinterpret_cast<uint4*>(smem + C::OFF_BIAS_A);
    for (int q = threadIdx.x; q < kBiasABytes / 16; q += blockDim.x) {
      const bool k_lo = ((q >> 3) & 1) == 0;          // 16-byte row chunk of K half 0 (elements 0..7)
      ba[q] = k_lo ? make_uint4(0x3F803F80u, 0x3F80u, 0u, 0u) : make_uint4(0u, 0u, 0u, 0u);
    }
    uint4* bb = reinterpret_cast<uint4*>(smem + C::OFF_BIAS_B);
    for (int q = threadIdx.x; q < TC_NBB * kBiasBBytes / 16; q += blockDim.x) bb[q] = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == TC_PRODUCER_WARP && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the next half-step may start its prologue, TMA loads and MMAs (which read only
  // the packed clouds) on SMs this grid has left; its bias warp waits for this grid's completion before reading
  // the potential this grid writes, and everything it writes waits on that bias.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const long long u_begin = sk_unit_begin(blockIdx.x, sk.units, sk.grid);
  const long long u_end = sk_unit_begin(blockIdx.x + 1, sk.units, sk.grid);
  const int dk = args.dk;
  const int ksteps = dk / 16;

  if (warp == TC_PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer
    int T = 0, seg = 0, seg_issued = 0;
    bool ok = true, issued_current = false;
    const TcColumnOrder order = tc_column_order<kRotate>(sk, u_begin, lane);
    for (long long u = u_begin; u < u_end && ok; ++seg) {
      const int r = (int)(u / sk.nct);
      const long long row_end = (long long)(r + 1) * sk.nct;
      const long long seg_end = min(u_end, row_end);
      const int rot = order.of_row(row_end, u_end);
      const int a_slot = seg & 1;
      ok = mbar_wait(&a_empty[a_slot], ((seg >> 1) & 1) ^ 1, abort_flag, p.error_word);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&a_full[a_slot], C::A_BYTES);
        for (int kb = 0; kb < NKB; ++kb)
          tma_load_2d(smem + a_slot * C::A_BYTES + kb * TC_BM * 128, &map_a, &a_full[a_slot], kb * 64, r * TC_BM);
      }
      seg_issued = seg + 1;
      for (; u < seg_end; ++u, ++T) {
        int c = (int)(u - (long long)r * sk.nct) + rot;   // (no 64-bit division per tile)
        if (kRotate && c >= sk.nct) c -= sk.nct;
        const int stage = T % C::NS;
        issued_current = false;
        ok = mbar_wait(&empty_b[stage], ((T / C::NS) & 1) ^ 1, abort_flag, p.error_word);
        if (!ok) break;
        issued_current = true;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full_b[stage], C::B_BYTES);
          for (int kb = 0; kb < NKB; ++kb)
            tma_load_2d(smem + C::OFF_B + stage * C::B_BYTES + kb * TC_BN * 128, &map_b, &full_b[stage], kb * 64,
                        c * TC_BN);
        }
      }
    }
    // Unwind: make sure no copy of ours is still landing in shared memory when the CTA exits. Stage s has had
    // ceil((issued - s) / NS) fills; the last one completes phase (fills - 1).
    if (!ok && lane == 0) {
      const int issued = T + (issued_current ? 1 : 0);
      for (int s = 0; s < C::NS; ++s) {
        const int fills = (issued - s + C::NS - 1) / C::NS;
        if (fills > 0) mbar_wait(&full_b[s], (uint32_t)((fills - 1) & 1), abort_flag, p.error_word, true);
      }
      for (int a = 0; a < 2; ++a) {
        const int fills = (seg_issued - a + 1) / 2;
        if (fills > 0) mbar_wait(&a_full[a], (uint32_t)((fills - 1) & 1), abort_flag, p.error_word, true);
      }
    }
  } else if (warp == TC_BIAS_WARP) {
    // ---------------------------------------------------------------- column bias operand
    // bias_j = (gh_j / eps + log b_j) log2(e), stored as bias_j / dot2 in three BF16 parts (K = 0, 1, 2 of row j
    // of the slot's B operand). All loads of a tile are issued before waiting for the slot, so a tile costs one
    // L2 round trip, overlapped with the MMAs of the tile before.
    const float* __restrict__ ghp = p.gh;
    const float* __restrict__ lbp = p.log_b;
    const float inv_dot2 = 1.0f / dot2_e;
    // The column tile is tracked, not divided out of u, and whole tiles load without bounds checks: this warp's
    // instructions share issue slots with the epilogue warps of its sub-partition.
    const TcColumnOrder order = tc_column_order<kRotate>(sk, u_begin, lane);
    int cu = order.phase;   // u mod nct
    long long row_end = u_begin - cu + sk.nct;
    int rot = order.of_row(row_end, u_end);
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the previous grid (which may write gh) is complete
    int T = 0;
    bool ok = true;
    if (args.pub.world > 1) {
      // gh is complete once every other GPU has published its rows of it (their stores land in this GPU's copy;
      // the loads below go through L2, never a stale L1 line)
      if (!wait_peers(args.pub, p.error_word)) {
        *abort_flag = 1;
        ok = false;
      }
    }
    for (long long u = u_begin; u < u_end && ok; ++u, ++T) {
      int c = cu + rot;
      if (kRotate && c >= sk.nct) c -= sk.nct;
      if (++cu == sk.nct) {
        cu = 0;
        row_end += sk.nct;
        rot = order.of_row(row_end, u_end);
      }
      float g[TC_BN / 32], l[TC_BN / 32];
      if ((c + 1) * TC_BN <= p.m) {
#pragma unroll
        for (int q = 0; q < TC_BN / 32; ++q) {
          const int j = c * TC_BN + q * 32 + lane;
          g[q] = __ldcg(ghp + j);
          l[q] = __ldg(lbp + j);
        }
      } else {
#pragma unroll
        for (int q = 0; q < TC_BN / 32; ++q) {
          const int j = c * TC_BN + q * 32 + lane;
          g[q] = j < p.m ? __ldcg(ghp + j) : 0.f;
          l[q] = j < p.m ? __ldg(lbp + j) : -INFINITY;
        }
      }
      const int bslot = T % TC_NBB;
      ok = mbar_wait(&bias_empty[bslot], ((T / TC_NBB) & 1) ^ 1, abort_flag, p.error_word);
      if (!ok) break;
      uint8_t* bb = smem + C::OFF_BIAS_B + bslot * kBiasBBytes;
#pragma unroll
      for (int q = 0; q < TC_BN / 32; ++q) {
        const float x = fmaf(l[q], p.lb2, g[q] * gh2_e) * inv_dot2;
        *reinterpret_cast<uint2*>(bb + bias_row_offset(q * 32 + lane)) =
            bias_split(fminf(fmaxf(x, -1e36f), 1e36f) + (x == -INFINITY ? -INFINITY : 0.f));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&bias_full[bslot]);
    }
  } else if (warp == TC_MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int T = 0, seg = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem);
      const uint32_t b_base = smem_u32(smem + C::OFF_B);
      const uint32_t bias_a = smem_u32(smem + C::OFF_BIAS_A);
      const uint32_t bias_b = smem_u32(smem + C::OFF_BIAS_B);
      const bool mirror = args.mirror != 0;
      for (long long u = u_begin; u < u_end && ok; ++seg) {
        const int r = (int)(u / sk.nct);
        const long long seg_end = min(u_end, (long long)(r + 1) * sk.nct);
        const int a_slot = seg & 1;
        ok = mbar_wait(&a_full[a_slot], (seg >> 1) & 1, abort_flag, p.error_word);
        if (!ok) break;
        for (; u < seg_end; ++u, ++T) {
          const int stage = T % C::NS;
          const int acc = T % TC_NACC;
          ok = mbar_wait(&acc_empty[acc], ((T / TC_NACC) & 1) ^ 1, abort_flag, p.error_word);
          if (ok) ok = mbar_wait(&full_b[stage], (T / C::NS) & 1, abort_flag, p.error_word);
          if (!ok) break;
          tmem_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * TC_BN);
          const uint32_t a_tile = a_base + a_slot * C::A_BYTES;
          const uint32_t b_tile = b_base + stage * C::B_BYTES;
          uint32_t accumulate = 0;
#pragma unroll
          for (int pass = 0; pass < 3; ++pass) {
            // The small correction products first, then hi.hi, in an order fixed by the two clouds rather than by
            // their roles: P_hi.Q_lo, P_lo.Q_hi, P_hi.Q_hi with P the cloud at the lower address. The f half-step
            // (x rows) and the g half-step (y rows) then accumulate x_i . y_j from the same products in the same
            // order, identically rounded (the tensor cores round the accumulation toward zero). With the order tied
            // to the roles the two half-steps see costs that differ in the last bits, and that difference drives the
            // nearly free relative potential of mutually dominant point pairs a little further every iteration.
            const int first = mirror ? 1 : 0;
            const int ea0 = (pass == 1 - first) ? dk : 0;
            const int eb0 = (pass == first) ? dk : 0;
            for (int kk = 0; kk < ksteps; ++kk) {
              const int ea = ea0 + 16 * kk, eb = eb0 + 16 * kk;
              const uint32_t sa = a_tile + (ea >> 6) * (TC_BM * 128) + (ea & 63) * 2;
              const uint32_t sb = b_tile + (eb >> 6) * (TC_BN * 128) + (eb & 63) * 2;
              umma_f16(d_tmem, sw128_desc(sa), sw128_desc(sb), kIdesc, accumulate);
              accumulate = 1;
            }
          }
          umma_commit(&empty_b[stage]);
          // last, the column bias (it is the only input that waits for the previous grid)
          const int bslot = T % TC_NBB;
          ok = mbar_wait(&bias_full[bslot], (T / TC_NBB) & 1, abort_flag, p.error_word);
          if (!ok) break;
          tmem_fence_after();
          umma_f16(d_tmem, plain_desc(bias_a, kBiasLbo, kBiasSbo),
                   plain_desc(bias_b + (uint32_t)(bslot * kBiasBBytes), kBiasLbo, kBiasSbo), kIdescBf16, 1u);
          umma_commit(&bias_empty[bslot]);
          umma_commit(&acc_full[acc]);
        }
        if (ok) umma_commit(&a_empty[a_slot]);
      }
      // Wait for every MMA we issued before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, abort_flag, p.error_word, true);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue warpgroups 0 and 1
    // Both warpgroups work on every tile: warpgroup wg takes columns [128 wg, 128 wg + 128) of the tile's
    // accumulator and releases the accumulator as soon as its last TMEM read of the tile is done (inside
    // lse_tile128), so the MMAs two tiles ahead overlap the rest of the fold.
    const int wg = warp >> 2;
    const int qrow = (warp & 3) * 32 + lane;   // this thread's row in the tile == its TMEM lane
    const uint32_t lane_base = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(wg * (TC_BN / 2));
    const float dot2 = dot2_e;
    int T = 0;
    bool ok = true, published = false;
    // A segment's arrival on its row tile's counter is an acquire-release atomic by one thread after the warpgroup's
    // partial stores and a warpgroup barrier (the release covers the barrier's other threads' stores); its result
    // -- whether this warpgroup is the row tile's last arrival and merges it -- is looked at one tile later (or at
    // the end of the range), so the atomic's round trip to L2 overlaps the next tile's fold instead of stalling it.
    bool pending = false;
    int pend_old = 0;   // the atomic's result (thread qrow 0)
#define TRNOPT_RESOLVE_ARRIVAL(kWide)                                                                   \
  do {                                                                                                  \
    if (qrow == 0) s_last[wg] = (pend_old == s_pend[2 * wg + 1] - 1);                                   \
    asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");                                         \
    if (s_last[wg]) {                                                                                   \
      const int pend_r = s_pend[2 * wg], pend_expected = s_pend[2 * wg + 1];                             \
      const int row = pend_r * TC_BM + qrow;                                                            \
      if (row < p.rows) {                                                                               \
        const float2* base = sk.partials + (size_t)pend_r * sk.slots * TC_BM;                           \
        const float v = finish_row<kWide>(p, row, base + qrow, pend_expected, TC_BM, eps_e, kappa_e);   \
        if (args.pub.world > 1) {                                                                       \
          publish_row(args.pub, row, v);                                                                \
          published = true;                                                                             \
        }                                                                                               \
      }                                                                                                 \
      if (qrow == 0) sk.counters[pend_r] = 0;                                                           \
    }                                                                                                   \
    asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory"); /* s_last read before its next write */ \
    pending = false;                                                                                    \
  } while (0)
    for (long long u = u_begin; u < u_end;) {
      const int r = (int)(u / sk.nct);
      const long long seg_end = min(u_end, (long long)(r + 1) * sk.nct);
      float M = kMaxFloor, L = 0.f;
      for (; u < seg_end; ++u, ++T) {
        if (ok) {
          const int acc = T % TC_NACC;
          // (one decision per warp: the tile's TMEM loads are warp-collective)
          ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (T / TC_NACC) & 1, abort_flag, p.error_word));
          if (ok) {
            tmem_fence_after();
            lse_tile128(lane_base + (uint32_t)(acc * TC_BN), dot2, M, L, &acc_empty[acc]);
          }
        }
        if (pending) TRNOPT_RESOLVE_ARRIVAL(false);
      }
      // Segment done: this warpgroup's partial for row tile r, then one arrival on the row tile's counter.
      const long long first_u = (long long)r * sk.nct;
      const int kfirst = sk_cta_of(first_u, sk.units, sk.grid);
      const int klast = sk_cta_of(first_u + sk.nct - 1, sk.units, sk.grid);
      const int expected = 2 * (klast - kfirst + 1);
      const int slot = 2 * (blockIdx.x - kfirst) + wg;
      sk.partials[((size_t)r * sk.slots + slot) * TC_BM + qrow] = make_float2(M, L);
      asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
      if (qrow == 0) {
        s_pend[2 * wg] = r;
        s_pend[2 * wg + 1] = expected;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(pend_old) : "l"(sk.counters + r) : "memory");
      }
      pending = true;
    }
    // The end of the range: nothing overlaps this merge. Row tiles spread over many CTAs (small problems) read their
    // partials in one round of loads, in the one-K-block kernel (d <= 32: the single-cell pairs); in the two-K-block
    // kernel the extra code measured 0.8 % slower at config 2, whose merges never need it.
    if (pending) TRNOPT_RESOLVE_ARRIVAL(NKB == 1);
#undef TRNOPT_RESOLVE_ARRIVAL
    if (published) __threadfence_system();   // this thread's peer stores, before the CTA barrier below
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == TC_MMA_WARP) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
  }
  if (args.pub.world > 1 && threadIdx.x == 0) publish_done(args.pub);
}

// ------------------------------------------------------------------------------------------------------------
// Packing: rows of [hi (dk) | lo (dk) | zero padding to kp] in FP16 from transposed FP32 points.
// ------------------------------------------------------------------------------------------------------------

__global__ void tc_pack_kernel(const float* __restrict__ xT, int ldx, int n, int d, int dk, int kp, float scale,
                               __half* __restrict__ out) {
  const long long total = (long long)n * kp;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx / kp), k = (int)(idx % kp);
    __half h = __float2half_rn(0.f);
    const int kk = k < dk ? k : k - dk;
    if (k < 2 * dk && kk < d) {
      const float v = xT[(size_t)kk * ldx + i] * scale;     // exact: scale is a power of two
      const __half hi = __float2half_rn(v);
      h = (k < dk) ? hi : __float2half_rn(v - __half2float(hi));
    }
    out[idx] = h;
  }
}

__global__ void ex2_poly_kernel(const float* __restrict__ x, float* __restrict__ out, int n) {
  // (through the packed pair form the fold uses; NaN wherever its two lanes or the scalar form disagree)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float a, b;
    upk2(ex2_poly2(x[i], x[i]), a, b);
    out[i] = (__float_as_uint(a) == __float_as_uint(b) && __float_as_uint(a) == __float_as_uint(ex2_poly(x[i])))
                 ? a
                 : __int_as_float(0x7fc00000);   // NaN: the test sees it
  }
}

cudaError_t ex2_poly_launch(const float* x, float* out, int n, cudaStream_t stream) {
  ex2_poly_kernel<<<(n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184, 256, 0, stream>>>(x, out, n);
  return cudaGetLastError();
}

int tc_dk(int d) { return (d + 15) / 16 * 16; }
int tc_kp(int d) { return (2 * tc_dk(d) + 63) / 64 * 64; }
int tc_supported_d(int d) { return (d >= 1 && tc_kp(d) <= 128) ? tc_dk(d) : 0; }

cudaError_t tc_pack(const float* xT, int ldx, int n, int d, int scale_exp, void* packed, cudaStream_t stream) {
  const int dk = tc_dk(d), kp = tc_kp(d);
  const long long total = (long long)n * kp;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  tc_pack_kernel<<<grid, threads, 0, stream>>>(xT, ldx, n, d, dk, kp, ldexpf(1.0f, scale_exp),
                                               reinterpret_cast<__half*>(packed));
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------
// Host side: tensor maps (cached per pointer / shape), planning, launch
// ------------------------------------------------------------------------------------------------------------

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

struct MapEntry {
  const void* ptr;
  int rows, kp, box_rows;
  CUtensorMap map;
};
constexpr int kMapCache = 32;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mutex;

bool tensor_map(const void* ptr, int rows, int kp, int box_rows, CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mutex);
  for (int i = 0; i < kMapCache; ++i) {
    const MapEntry& e = g_maps[i];
    if (e.ptr == ptr && e.rows == rows && e.kp == kp && e.box_rows == box_rows) {
      *out = e.map;
      return true;
    }
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  MapEntry e{ptr, rows, kp, box_rows, {}};
  const cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kp * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&e.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  g_maps[g_map_next] = e;
  g_map_next = (g_map_next + 1) % kMapCache;
  *out = e.map;
  return true;
}

int g_tc_sms[64] = {0};

}  // namespace

// Column clouds above this size (packed FP16 bytes) are swept in the CTAs' common phase (tc_column_order).
constexpr long long kTcRotateBytes = 32ll << 20;

void tc_plan(int device, int rows, int m, int d, StreamK& sk) {
  if (device < 0 || device >= 64) device = 0;
  if (g_tc_sms[device] == 0) cudaDeviceGetAttribute(&g_tc_sms[device], cudaDevAttrMultiProcessorCount, device);
  sk.nrt = (rows + TC_BM - 1) / TC_BM;
  sk.nct = (m + TC_BN - 1) / TC_BN;
  sk.units = (long long)sk.nrt * sk.nct;
  const long long g = g_tc_sms[device] > 0 ? g_tc_sms[device] : 148;
  sk.grid = (int)(g < sk.units ? g : sk.units);
  sk.slots = 2 * sk_max_slots(sk.units, sk.grid, sk.nct);
  sk.parts_per_cta = 2;
  sk.rotate = (long long)m * tc_kp(d) * 2 > kTcRotateBytes ? 1 : 0;
}

size_t tc_partial_bytes(const StreamK& sk) { return (size_t)sk.nrt * sk.slots * TC_BM * sizeof(float2); }

template <int NKB, bool kRotate>
static cudaError_t tc_launch_t(const CUtensorMap& ma, const CUtensorMap& mb, const TcArgs& a, cudaStream_t stream,
                               bool pdl) {
  using C = TcCfg<NKB>;
  static std::atomic<int> attr_done[kMaxDevices];
  cudaError_t e =
      smem_attr_once(reinterpret_cast<const void*>(half_step_tc_kernel<NKB, kRotate>), C::SMEM, attr_done);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.sk.grid);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, half_step_tc_kernel<NKB, kRotate>, ma, mb, a);
}

cudaError_t tc_launch(const LseProblem& p, const void* xpack, const void* ypack, int sx, int sy, const StreamK& sk,
                      cudaStream_t stream, const Publish* pub, bool pdl) {
  const int kp = tc_kp(p.d);
  CUtensorMap ma, mb;
  if (!tensor_map(xpack, p.rows, kp, TC_BM, &ma) || !tensor_map(ypack, p.m, kp, TC_BN, &mb))
    return cudaErrorInvalidValue;
  TcArgs a;
  a.p = p;
  a.dot2_scale = (float)ldexp(1.0, -(sx + sy));
  a.mirror = reinterpret_cast<uintptr_t>(xpack) > reinterpret_cast<uintptr_t>(ypack);
  a.p.dot2 = (float)((double)p.dot2 * ldexp(1.0, -(sx + sy)));
  a.sk = sk;
  a.dk = tc_dk(p.d);
  if (pub) {
    a.pub = *pub;
  } else {
    a.pub = Publish{};
    a.pub.world = 1;
  }
  // (the rotation is a template choice: the kernel without it carries none of its code)
  if (kp == 64) {
    return sk.rotate ? tc_launch_t<1, true>(ma, mb, a, stream, pdl) : tc_launch_t<1, false>(ma, mb, a, stream, pdl);
  }
  return sk.rotate ? tc_launch_t<2, true>(ma, mb, a, stream, pdl) : tc_launch_t<2, false>(ma, mb, a, stream, pdl);
}

}  // namespace trnopt
