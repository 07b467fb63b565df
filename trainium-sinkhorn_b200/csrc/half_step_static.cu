// trnopt_half_step_tc_static: the tensor-core half-step for callers that cannot allocate device memory.
//
// Some callers of this library have no way to call cudaMalloc: code running inside a CUDA graph that is being
// captured by someone else, plugin hosts that hand out only the input and output buffers, and allocators that
// forbid allocations after start-up (an arena sized once at launch). For them this entry point takes the same
// inputs and outputs as trnopt_half_step_tc and keeps its scratch (the per-row-tile arrival counters, then the
// per-row partial maxima/sums) in a fixed array compiled into the library instead of a caller workspace.
//
// Limits and sharing:
//   * The array is kStaticScratchBytes (4 MiB) per GPU, held from the moment the library is loaded on that GPU until
//     the process exits. Problems whose scratch need (trnopt_workspace_size(rows, m, d, TRNOPT_PATH_TC)) exceeds it
//     are rejected with TRNOPT_ERR_TOO_LARGE before anything is enqueued. The need grows with the row tiles and
//     with the stream-K split, which depends on the GPU's SM count, so the largest problem that fits depends on the
//     device: on a 148-SM B200, 10k x 10k needs about 0.5 MB and 100k x 100k about 3.2 MB. Callers check
//     trnopt_workspace_size against trnopt_static_scratch_bytes() on their own device.
//   * Every call on a GPU uses the same array, which keeps whatever the last call left in it. The counters that must
//     start at zero are cleared (cudaMemsetAsync on the array, no allocation) at the start of every call. Calls
//     whose kernels can overlap on the GPU (different streams, or several host threads) race on the array and
//     give wrong results: serialise them on one stream.
//   * The array's name is a host-side stand-in in host code, not a device address. Its device address is looked
//     up once per GPU, with that GPU current, by the first call made on it (cudaGetSymbolAddress); make that first
//     call before any stream capture begins on that GPU.
#include <mutex>

#include "../../include/trnopt_cuda.h"
#include "kernels.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
using trnopt::kMaxDevices;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the static array on the current GPU (looked up once per GPU).
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return TRNOPT_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return TRNOPT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) return TRNOPT_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TRNOPT_OK;
}

}  // namespace

extern "C" {

size_t trnopt_static_scratch_bytes(void) { return kStaticScratchBytes; }

int trnopt_half_step_tc_static(const void* xpack, const float* xsq, const float* off, const void* ypack,
                               const float* gh, const float* log_b, int rows, int m, int d, int sx, int sy, float eps,
                               float kappa, float* fh, void* stream) {
  // Every check that trnopt_half_step_tc makes, before anything is enqueued: a rejected call leaves nothing on the
  // caller's stream (no stray memset node in a graph the caller is capturing).
  int st = trnopt::half_step_tc_check(xpack, xsq, ypack, gh, log_b, rows, m, d, eps, kappa, fh);
  if (st != TRNOPT_OK) return st;
  const size_t need = trnopt_workspace_size(rows, m, d, TRNOPT_PATH_TC);
  if (need == 0) return TRNOPT_ERR_UNSUPPORTED;
  if (need > kStaticScratchBytes) return TRNOPT_ERR_TOO_LARGE;
  void* scratch = nullptr;
  st = static_scratch(&scratch);
  if (st != TRNOPT_OK) return st;
  // The arrival counters (one int per 128-row tile, at the start of the scratch) must start at zero.
  const size_t counters = ((size_t)(rows + 127) / 128 * sizeof(int) + 255) / 256 * 256;
  if (cudaMemsetAsync(scratch, 0, counters, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return TRNOPT_ERR_CUDA;
  return trnopt_half_step_tc(xpack, xsq, off, ypack, gh, log_b, rows, m, d, sx, sy, eps, kappa, fh, scratch,
                             kStaticScratchBytes, stream);
}

}  // extern "C"
