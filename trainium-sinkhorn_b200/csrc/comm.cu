// A device region shared by the GPUs of one job (one process per GPU), mapped into every other process with CUDA IPC,
// and the sharded Sinkhorn run that uses it.
//
// Each rank allocates one region: a 256-byte header (the flag array, one 64-bit slot per rank, and a CTA counter)
// followed by the caller's buffers. The ranks exchange IPC handles (through the caller's process group) and map one
// another's regions, so the same buffer offset names "this vector" on every GPU. A half-step run with a Publish
// (common.cuh) stores its rows into the vector on every GPU and then raises this rank's flag on every GPU to the
// launch's epoch; the next half-step on any GPU reads its input once every other rank's flag shows the epoch it
// depends on. This replaces the all-gather after each half-step (the reference exchanges the half-step's blocks
// between NeuronCores through the host, src/trnopt/sinkhorn.py:295-311): the rows cross NVLink while the epilogue
// runs, and no collective launch or host step sits between half-steps.
//
// Epochs count published launches (and arrivals, below) and advance identically on every rank, because every rank
// makes the same calls in the same order.
#include <stdint.h>
#include <string.h>

#include "../../include/trnopt_cuda.h"
#include "kernels.h"

namespace trnopt {
namespace {

constexpr size_t kCommHeader = 256;   // flags[kMaxRanks] (u64) at 0, CTA counter (int) at 64

struct Comm {
  int rank = 0, world = 1, device = 0;
  size_t bytes = 0;                    // caller's bytes after the header
  char* base = nullptr;                // this rank's region
  char* peer_base[kMaxRanks] = {};     // every rank's region as mapped here (peer_base[rank] == base)
  bool open = false;
  unsigned long long epoch = 0;        // last epoch this rank has published
};

unsigned long long* flags_of(char* region) { return reinterpret_cast<unsigned long long*>(region); }

// Raise this rank's slot on every other GPU to `epoch` once everything queued before on the stream is done.
__global__ void comm_arrive_kernel(Publish pub) {
  __threadfence_system();
  for (int q = 0; q < pub.world; ++q)
    if (q != pub.rank) st_release_sys(pub.flag_peer[q], pub.epoch);
}

// Hold the stream until every other rank's slot reaches pub.wait_epoch (one warp; bounded, kErrPeerTimeout on
// expiry).
__global__ void comm_wait_kernel(Publish pub, int* error_word) { wait_peers(pub, error_word); }

Publish make_publish(const Comm& c, const float* out) {
  Publish p{};
  p.world = c.world;
  p.rank = c.rank;
  const ptrdiff_t off = reinterpret_cast<const char*>(out) - c.base;
  for (int q = 0; q < c.world; ++q) {
    p.out_peer[q] = out ? reinterpret_cast<float*>(c.peer_base[q] + off) : nullptr;
    p.flag_peer[q] = flags_of(c.peer_base[q]) + c.rank;
  }
  p.flags = flags_of(c.base);
  p.done = reinterpret_cast<int*>(c.base + 64);
  return p;
}

bool in_region(const Comm& c, const void* p, size_t bytes) {
  const char* b = static_cast<const char*>(p);
  return b >= c.base + kCommHeader && b + bytes <= c.base + kCommHeader + c.bytes;
}

int status_of(cudaError_t e) { return e == cudaSuccess ? TRNOPT_OK : TRNOPT_ERR_CUDA; }

}  // namespace
}  // namespace trnopt

using namespace trnopt;

extern "C" {

size_t trnopt_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int trnopt_comm_create(int rank, int world, size_t bytes, void** comm_out, void* handle_out) {
  if (!comm_out || !handle_out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || bytes == 0)
    return TRNOPT_ERR_INVALID_ARGUMENT;
  *comm_out = nullptr;
  Comm* c = new Comm;
  c->rank = rank;
  c->world = world;
  c->bytes = (bytes + 255) / 256 * 256;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->base), kCommHeader + c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, kCommHeader + c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), c->base);
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    delete c;
    return TRNOPT_ERR_CUDA;
  }
  c->peer_base[rank] = c->base;
  *comm_out = c;
  return TRNOPT_OK;
}

int trnopt_comm_open(void* comm, const void* handles) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !handles || c->open) return TRNOPT_ERR_INVALID_ARGUMENT;
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int k = 0; k < q; ++k)
        if (k != c->rank && c->peer_base[k]) {
          cudaIpcCloseMemHandle(c->peer_base[k]);
          c->peer_base[k] = nullptr;
        }
      return TRNOPT_ERR_CUDA;
    }
    c->peer_base[q] = static_cast<char*>(p);
  }
  c->open = true;
  return TRNOPT_OK;
}

void* trnopt_comm_buffer(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  return c ? c->base + kCommHeader : nullptr;
}

size_t trnopt_comm_buffer_bytes(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  return c ? c->bytes : 0;
}

unsigned long long trnopt_comm_epoch(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  return c ? c->epoch : 0;
}

int trnopt_comm_arrive(void* comm, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || (c->world > 1 && !c->open)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (c->world == 1) return TRNOPT_OK;
  Publish p = make_publish(*c, nullptr);
  p.epoch = c->epoch + 1;
  comm_arrive_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) c->epoch = p.epoch;
  return status_of(e);
}

int trnopt_comm_wait(void* comm, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || (c->world > 1 && !c->open)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (c->world == 1) return TRNOPT_OK;
  Publish p = make_publish(*c, nullptr);
  p.wait_epoch = c->epoch;
  comm_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p, device_error_word());
  return status_of(cudaGetLastError());
}

int trnopt_comm_destroy(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return TRNOPT_ERR_INVALID_ARGUMENT;
  int st = TRNOPT_OK;
  for (int q = 0; q < c->world; ++q)
    if (q != c->rank && c->peer_base[q] && cudaIpcCloseMemHandle(c->peer_base[q]) != cudaSuccess) st = TRNOPT_ERR_CUDA;
  if (c->base && cudaFree(c->base) != cudaSuccess) st = TRNOPT_ERR_CUDA;
  delete c;
  return st;
}

int trnopt_sinkhorn_run_sharded(void* comm, const void* xpack, const float* xsq, const float* xoff,
                                const float* log_a, int nx, int sx, const void* ypack, const float* ysq,
                                const float* yoff, const float* log_b, int ny, int sy, int d, float* g0, float* g1,
                                float* fh, int start_parity, int n_iter, float eps, float kappa_x, float kappa_y,
                                void* workspace, size_t ws_bytes, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || n_iter < 0 || !xpack || !ypack || !xsq || !ysq || !log_a || !log_b || !g0 || !g1 || !fh)
    return TRNOPT_ERR_INVALID_ARGUMENT;
  const int W = c->world, r = c->rank;
  if (W > 1 && !c->open) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (nx < 1 || ny < 1 || nx % (128 * W) || ny % (128 * W)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!tc_supported_d(d)) return TRNOPT_ERR_UNSUPPORTED;
  if (!in_region(*c, g0, (size_t)ny * 4) || !in_region(*c, g1, (size_t)ny * 4) || !in_region(*c, fh, (size_t)nx * 4))
    return TRNOPT_ERR_INVALID_ARGUMENT;
  const size_t row_bytes = (size_t)tc_kp(d) * 2;
  const int sxr = nx / W, syr = ny / W, x0 = r * sxr, y0 = r * syr;
  const void* xp = static_cast<const char*>(xpack) + (size_t)x0 * row_bytes;
  const void* yp = static_cast<const char*>(ypack) + (size_t)y0 * row_bytes;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_iter; ++i) {
    float* gc = ((start_parity + i) & 1) ? g1 : g0;
    float* gn = ((start_parity + i) & 1) ? g0 : g1;
    Publish pf = make_publish(*c, fh + x0);
    pf.wait_epoch = c->epoch;
    pf.epoch = c->epoch + 1;
    int st = half_step_tc_launch(xp, xsq + x0, xoff ? xoff + x0 : nullptr, ypack, gc, log_b, sxr, ny, d, sx, sy, eps,
                                 kappa_x, fh + x0, workspace, ws_bytes, s, W > 1 ? &pf : nullptr);
    if (st != TRNOPT_OK) return st;
    c->epoch = pf.epoch;
    Publish pg = make_publish(*c, gn + y0);
    pg.wait_epoch = c->epoch;
    pg.epoch = c->epoch + 1;
    st = half_step_tc_launch(yp, ysq + y0, yoff ? yoff + y0 : nullptr, xpack, fh, log_a, syr, nx, d, sy, sx, eps,
                             kappa_y, gn + y0, workspace, ws_bytes, s, W > 1 ? &pg : nullptr, nullptr, 1, true);
    if (st != TRNOPT_OK) return st;
    c->epoch = pg.epoch;
  }
  return TRNOPT_OK;
}

}  // extern "C"
