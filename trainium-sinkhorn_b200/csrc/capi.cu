// C ABI of libtrnopt_cuda.so: argument checks, workspace layout and dispatch to the kernels.
// The declarations, with the reference interface each entry point replaces, are in include/trnopt_cuda.h.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/trnopt_cuda.h"
#include "kernels.h"

namespace trnopt {

__device__ int g_error_word;

// Per-device lookups cached once per device (the launch path queries them on every half-step).
namespace {
int* g_error_ptr[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
}  // namespace

int* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  if (g_error_ptr[dev] == nullptr) {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_error_word) == cudaSuccess) g_error_ptr[dev] = p;
    return p;
  }
  return g_error_ptr[dev];
}

int device_cc_major(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 0;
  if (g_cc_major[dev] == 0) cudaDeviceGetAttribute(&g_cc_major[dev], cudaDevAttrComputeCapabilityMajor, dev);
  return g_cc_major[dev];
}

}  // namespace trnopt

using namespace trnopt;

namespace {

thread_local int t_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return TRNOPT_OK;
  t_last_cuda_error = (int)e;
  return TRNOPT_ERR_CUDA;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr size_t kCounterRegion = 256;   // bytes reserved per 64 row tiles for the arrival counters

size_t counter_bytes(int nrt) { return ((size_t)nrt * sizeof(int) + kCounterRegion - 1) / kCounterRegion * kCounterRegion; }

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// Counters region at the start of a workspace of ws_bytes: one int per KB of workspace. No call can have more row
// tiles than that (each row tile needs at least one 1 KB block of partials), and the size depends on ws_bytes
// only, so every call sharing a workspace (the f and g half-steps of a solve, of different shapes) puts its partials
// at the same offset, past every call's counters: a call's partials never overwrite another call's counters, and
// counters that calls share are zero between launches (every launch re-arms the counters it uses).
size_t counter_region(size_t ws_bytes) {
  return ((ws_bytes / 1024) * sizeof(int) + kCounterRegion - 1) / kCounterRegion * kCounterRegion;
}

// Smallest workspace that holds `partial_bytes` of partials past its counter region, for nrt row tiles.
size_t workspace_bytes(size_t partial_bytes, int nrt) {
  size_t w = partial_bytes + counter_bytes(nrt);
  while (counter_region(w) + partial_bytes > w || counter_region(w) < counter_bytes(nrt)) w += kCounterRegion;
  return w;
}

int bind_workspace(StreamK& sk, size_t partial_bytes, void* ws, size_t ws_bytes) {
  const size_t region = counter_region(ws_bytes);
  if (ws == nullptr || counter_bytes(sk.nrt) > region || region + partial_bytes > ws_bytes)
    return TRNOPT_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return TRNOPT_ERR_ALIGNMENT;
  sk.counters = reinterpret_cast<int*>(ws);
  sk.partials = reinterpret_cast<float2*>(reinterpret_cast<char*>(ws) + region);
  return TRNOPT_OK;
}

int check_points(const float* pT, int ld, int count, int d) {
  if (pT == nullptr || count < 1 || d < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (ld < count) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (ld % 4 != 0 || !aligned(pT, 16)) return TRNOPT_ERR_ALIGNMENT;
  return TRNOPT_OK;
}

int ffma_run(LseProblem& p, void* ws, size_t ws_bytes, cudaStream_t stream) {
  StreamK sk{};
  ffma_plan(current_device(), p.rows, p.m, p.d, sk);
  int st = bind_workspace(sk, ffma_partial_bytes(sk), ws, ws_bytes);
  if (st != TRNOPT_OK) return st;
  p.error_word = device_error_word();
  return cuda_status(ffma_launch(p, sk, stream));
}

}  // namespace

namespace trnopt {

int half_step_tc_check(const void* xpack, const float* xsq, const void* ypack, const float* gh, const float* log_b,
                       int rows, int m, int d, float eps, float kappa, const float* fh) {
  if (!tc_supported_d(d)) return TRNOPT_ERR_UNSUPPORTED;
  if (!xpack || !ypack || !xsq || !gh || !log_b || !fh || rows < 1 || m < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned(xpack, 128) || !aligned(ypack, 128)) return TRNOPT_ERR_ALIGNMENT;
  if (!(eps > 0.f) || !isfinite(eps) || !isfinite(kappa)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (device_cc_major(current_device()) != 10) return TRNOPT_ERR_UNSUPPORTED;
  return TRNOPT_OK;
}

int half_step_tc_launch(const void* xpack, const float* xsq, const float* off, const void* ypack, const float* gh,
                        const float* log_b, int rows, int m, int d, int sx, int sy, float eps, float kappa, float* fh,
                        void* workspace, size_t ws_bytes, cudaStream_t stream, const Publish* pub,
                        const TrnoptSolveState* dyn, int side, bool pdl) {
  int st0 = half_step_tc_check(xpack, xsq, ypack, gh, log_b, rows, m, d, eps, kappa, fh);
  if (st0 != TRNOPT_OK) return st0;
  const int dev = current_device();
  LseProblem p{};
  p.gh = gh; p.log_b = log_b; p.xsq = xsq; p.off = off; p.rows = rows; p.m = m; p.d = d;
  const double inv_eps = 1.0 / (double)eps;
  p.dot2 = (float)(2.0 * inv_eps * 1.4426950408889634);
  p.gh2 = (float)(inv_eps * 1.4426950408889634);
  p.lb2 = kLog2e;
  p.eps = (double)eps; p.kappa = (double)kappa; p.mode = 0; p.out = fh;
  p.dyn = dyn; p.side = side;
  StreamK sk{};
  tc_plan(dev, rows, m, d, sk);
  int st = bind_workspace(sk, tc_partial_bytes(sk), workspace, ws_bytes);
  if (st != TRNOPT_OK) return st;
  p.error_word = device_error_word();
  return cuda_status(tc_launch(p, xpack, ypack, sx, sy, sk, stream, pub, pdl));
}

int half_step_ffma_launch(const float* xT, int ldx, const float* xsq, const float* off, const float* yT, int ldy,
                          const float* gh, const float* log_b, int rows, int m, int d, float eps, float kappa, float* fh,
                          void* workspace, size_t ws_bytes, cudaStream_t stream, const TrnoptSolveState* dyn,
                          int side) {
  if (d > 128) return TRNOPT_ERR_UNSUPPORTED;
  int st = check_points(xT, ldx, rows, d);
  if (st == TRNOPT_OK) st = check_points(yT, ldy, m, d);
  if (st != TRNOPT_OK) return st;
  if (xsq == nullptr || gh == nullptr || log_b == nullptr || fh == nullptr) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!(eps > 0.f) || !isfinite(eps) || !isfinite(kappa)) return TRNOPT_ERR_INVALID_ARGUMENT;
  LseProblem p{};
  p.xT = xT; p.ldx = ldx; p.yT = yT; p.ldy = ldy; p.gh = gh; p.log_b = log_b; p.xsq = xsq; p.off = off;
  p.rows = rows; p.m = m; p.d = d;
  const double inv_eps = 1.0 / (double)eps;
  p.dot2 = (float)(2.0 * inv_eps * 1.4426950408889634);
  p.gh2 = (float)(inv_eps * 1.4426950408889634);
  p.lb2 = kLog2e;
  p.eps = (double)eps; p.kappa = (double)kappa; p.mode = 0; p.out = fh;
  p.dyn = dyn; p.side = side;
  return ffma_run(p, workspace, ws_bytes, stream);
}

}  // namespace trnopt

extern "C" {

int trnopt_version(void) { return 100; }

const char* trnopt_status_string(int status) {
  switch (status) {
    case TRNOPT_OK: return "ok";
    case TRNOPT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TRNOPT_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case TRNOPT_ERR_WORKSPACE: return "workspace missing or too small";
    case TRNOPT_ERR_UNSUPPORTED: return "unsupported shape or path";
    case TRNOPT_ERR_CUDA: return "CUDA runtime error";
    case TRNOPT_ERR_DEVICE: return "a kernel reported an error flag";
    case TRNOPT_ERR_TOO_LARGE: return "problem needs more scratch than the static array of the no-allocation entry";
    default: return "unknown status";
  }
}

int trnopt_last_cuda_error(void) { return t_last_cuda_error; }

int trnopt_device_error_flags(void* stream, int* flags_out) {
  if (flags_out == nullptr) return TRNOPT_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int flags = 0;
  int st = cuda_status(cudaMemcpyFromSymbolAsync(&flags, g_error_word, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  if (st == TRNOPT_OK) st = cuda_status(cudaStreamSynchronize(s));
  if (st != TRNOPT_OK) return st;
  if (flags != 0) {
    const int zero = 0;
    st = cuda_status(cudaMemcpyToSymbolAsync(g_error_word, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    if (st == TRNOPT_OK) st = cuda_status(cudaStreamSynchronize(s));
  }
  *flags_out = flags;
  return st;
}

size_t trnopt_workspace_size(int rows, int m, int d, int path) {
  if (rows < 1 || m < 1 || d < 1) return 0;
  StreamK sk{};
  size_t partial = 0;
  if (path == TRNOPT_PATH_FFMA) {
    ffma_plan(current_device(), rows, m, d, sk);
    partial = ffma_partial_bytes(sk);
  } else if (path == TRNOPT_PATH_TC) {
    if (!tc_supported_d(d)) return 0;
    tc_plan(current_device(), rows, m, d, sk);
    partial = tc_partial_bytes(sk);
  } else {
    return 0;
  }
  return workspace_bytes(partial, sk.nrt);
}

int trnopt_workspace_init(void* workspace, size_t ws_bytes, void* stream) {
  if (workspace == nullptr || ws_bytes == 0) return TRNOPT_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaMemsetAsync(workspace, 0, ws_bytes, reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_half_step(const float* xT, int ldx, const float* xsq, const float* off, const float* yT, int ldy,
                     const float* gh, const float* log_b, int rows, int m, int d, float eps, float kappa, float* fh,
                     void* workspace, size_t ws_bytes, void* stream) {
  return half_step_ffma_launch(xT, ldx, xsq, off, yT, ldy, gh, log_b, rows, m, d, eps, kappa, fh, workspace, ws_bytes,
                               reinterpret_cast<cudaStream_t>(stream), nullptr, 0);
}

int trnopt_row_lse(const float* xaT, int ldx, const float* yaT, int ldy, int rows, int m, int k, float* lse,
                   void* workspace, size_t ws_bytes, void* stream) {
  if (k > 128) return TRNOPT_ERR_UNSUPPORTED;
  int st = check_points(xaT, ldx, rows, k);
  if (st == TRNOPT_OK) st = check_points(yaT, ldy, m, k);
  if (st != TRNOPT_OK) return st;
  if (lse == nullptr) return TRNOPT_ERR_INVALID_ARGUMENT;
  LseProblem p{};
  p.xT = xaT; p.ldx = ldx; p.yT = yaT; p.ldy = ldy; p.rows = rows; p.m = m; p.d = k;
  p.dot2 = kLog2e; p.gh2 = 0.f; p.lb2 = 0.f; p.eps = 1.0; p.kappa = 1.0; p.mode = 1; p.out = lse;
  return ffma_run(p, workspace, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t trnopt_pack_bytes(int n, int d) {
  if (n < 1 || !tc_supported_d(d)) return 0;
  return (size_t)n * tc_kp(d) * 2;
}

int trnopt_pack_cloud(const float* xT, int ldx, int n, int d, int scale_exp, void* packed, void* stream) {
  if (!tc_supported_d(d)) return TRNOPT_ERR_UNSUPPORTED;
  int st = check_points(xT, ldx, n, d);
  if (st != TRNOPT_OK) return st;
  if (packed == nullptr || scale_exp < -100 || scale_exp > 100) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned(packed, 128)) return TRNOPT_ERR_ALIGNMENT;
  return cuda_status(tc_pack(xT, ldx, n, d, scale_exp, packed, reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_half_step_tc(const void* xpack, const float* xsq, const float* off, const void* ypack, const float* gh,
                        const float* log_b, int rows, int m, int d, int sx, int sy, float eps, float kappa, float* fh,
                        void* workspace, size_t ws_bytes, void* stream) {
  return half_step_tc_launch(xpack, xsq, off, ypack, gh, log_b, rows, m, d, sx, sy, eps, kappa, fh, workspace,
                             ws_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

int trnopt_test_ex2_poly(const float* x, float* out, int n, void* stream) {
  if (!x || !out || n < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  return cuda_status(ex2_poly_launch(x, out, n, reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_sinkhorn_run(int path, const void* x_op, int ldx, const float* xsq, const float* xoff, const float* log_a,
                        int nx, int sx, const void* y_op, int ldy, const float* ysq, const float* yoff,
                        const float* log_b, int ny, int sy, int d, float* g0, float* g1, float* fh, int start_parity,
                        int n_iter, float eps, float kappa_x, float kappa_y, void* workspace, size_t ws_bytes,
                        void* stream) {
  if (n_iter < 0 || !g0 || !g1 || !fh) return TRNOPT_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < n_iter; ++i) {
    float* gc = ((start_parity + i) & 1) ? g1 : g0;
    float* gn = ((start_parity + i) & 1) ? g0 : g1;
    int st;
    if (path == TRNOPT_PATH_TC) {
      cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
      st = half_step_tc_launch(x_op, xsq, xoff, y_op, gc, log_b, nx, ny, d, sx, sy, eps, kappa_x, fh, workspace,
                               ws_bytes, s, nullptr, nullptr, 0, true);
      if (st == TRNOPT_OK)
        st = half_step_tc_launch(y_op, ysq, yoff, x_op, fh, log_a, ny, nx, d, sy, sx, eps, kappa_y, gn, workspace,
                                 ws_bytes, s, nullptr, nullptr, 1, true);
    } else if (path == TRNOPT_PATH_FFMA) {
      const float* xT = static_cast<const float*>(x_op);
      const float* yT = static_cast<const float*>(y_op);
      st = trnopt_half_step(xT, ldx, xsq, xoff, yT, ldy, gc, log_b, nx, ny, d, eps, kappa_x, fh, workspace, ws_bytes,
                            stream);
      if (st == TRNOPT_OK)
        st = trnopt_half_step(yT, ldy, ysq, yoff, xT, ldx, fh, log_a, ny, nx, d, eps, kappa_y, gn, workspace,
                              ws_bytes, stream);
    } else {
      st = TRNOPT_ERR_INVALID_ARGUMENT;
    }
    if (st != TRNOPT_OK) return st;
  }
  return TRNOPT_OK;
}

size_t trnopt_median_workspace_size(void) { return median_workspace_bytes(); }

int trnopt_median_cost(const double* xc, const double* yc, const double* sqx, const double* sqy, int n, int m, int d,
                       double* out, void* workspace, size_t ws_bytes, void* stream) {
  if (!xc || !yc || !sqx || !sqy || !out || n < 1 || m < 1 || d < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (d > 128) return TRNOPT_ERR_UNSUPPORTED;
  if ((long long)n * (long long)m > 100000000ll) return TRNOPT_ERR_UNSUPPORTED;
  if (workspace == nullptr || ws_bytes < median_workspace_bytes()) return TRNOPT_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(xc, 8) || !aligned(yc, 8)) return TRNOPT_ERR_ALIGNMENT;
  return cuda_status(median_launch(xc, yc, sqx, sqy, n, m, d, out, workspace, reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_balanced_error(const float* gh_old, const float* gh_new, const float* w, int n, float inv_eps,
                          float* out, void* stream) {
  if (!gh_old || !gh_new || !w || !out || n < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  return cuda_status(balanced_error_launch(gh_old, gh_new, w, n, inv_eps, out, reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_recenter(float* gh, int n, int npad, double* gauge, const void* state, void* stream) {
  if (!gh || !gauge || n < 1 || npad < n) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned(gauge, 8) || !aligned(state, 8)) return TRNOPT_ERR_ALIGNMENT;
  return cuda_status(recenter_launch(gh, n, npad, gauge, static_cast<const TrnoptSolveState*>(state),
                                     reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_solve_init(void* state, const double* stage_eps, int n_stages, double final_eps, double rho_x,
                      double rho_y, int check_every, int max_iters, int stage_max_iters, int fixed_iters,
                      int sched_len, float tol, float stage_tol, int n_real, int npad, int it0, void* stream) {
  if (!state || n_stages < 0 || n_stages > TRNOPT_MAX_STAGES || (n_stages > 0 && !stage_eps)) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!(final_eps > 0.0) || check_every < 1 || max_iters < 0 || n_real < 1 || npad < n_real || it0 < 0)
    return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned(state, 8)) return TRNOPT_ERR_ALIGNMENT;
  TrnoptSolveState h{};
  for (int k = 0; k < n_stages; ++k) {
    if (!(stage_eps[k] > 0.0)) return TRNOPT_ERR_INVALID_ARGUMENT;
    h.stage_eps[k] = stage_eps[k];
  }
  h.stage_eps[n_stages] = final_eps;
  h.rho[0] = rho_x;
  h.rho[1] = rho_y;
  h.tol = tol;
  h.stage_tol = stage_tol;
  h.n_stages = n_stages;
  h.check_every = check_every;
  h.max_iters = max_iters;
  h.stage_max_iters = stage_max_iters;
  h.fixed_iters = fixed_iters;
  h.balanced = rho_x < 0.0 && rho_y < 0.0;
  h.sched_len = sched_len;
  h.n_real = n_real;
  h.npad = npad;
  h.it = it0;
  h.stage_it = it0;
  h.done = it0 >= max_iters;
  h.err = nanf("");                  // no check yet
  solve_stage_params(h);
  return cuda_status(cudaMemcpyAsync(state, &h, sizeof(h), cudaMemcpyHostToDevice,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

int trnopt_sinkhorn_run_checked(int path, const void* x_op, int ldx, const float* xsq, const float* xoff,
                                const float* log_a, int nx, int sx, const void* y_op, int ldy, const float* ysq,
                                const float* yoff, const float* log_b, int ny, int sy, int d, float* g0, float* g1,
                                float* fh, int start_parity, int n_iter, void* state, const float* w_y,
                                void* workspace, size_t ws_bytes, void* stream) {
  if (n_iter < 1 || !g0 || !g1 || !fh || !state || !w_y) return TRNOPT_ERR_INVALID_ARGUMENT;
  if (!aligned(state, 8)) return TRNOPT_ERR_ALIGNMENT;
  const TrnoptSolveState* dyn = static_cast<const TrnoptSolveState*>(state);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // eps and kappa come from the state; the values given here only pass the argument checks
  const float eps = 1.0f, kappa = 1.0f;
  for (int i = 0; i < n_iter; ++i) {
    float* gc = ((start_parity + i) & 1) ? g1 : g0;
    float* gn = ((start_parity + i) & 1) ? g0 : g1;
    int st;
    if (path == TRNOPT_PATH_TC) {
      // the run's first half-step follows the previous check without overlap, so it sees the state that check wrote
      st = half_step_tc_launch(x_op, xsq, xoff, y_op, gc, log_b, nx, ny, d, sx, sy, eps, kappa, fh, workspace, ws_bytes,
                               s, nullptr, dyn, 0, i > 0);
      if (st == TRNOPT_OK)
        st = half_step_tc_launch(y_op, ysq, yoff, x_op, fh, log_a, ny, nx, d, sy, sx, eps, kappa, gn, workspace,
                                 ws_bytes, s, nullptr, dyn, 1, true);
    } else if (path == TRNOPT_PATH_FFMA) {
      const float* xT = static_cast<const float*>(x_op);
      const float* yT = static_cast<const float*>(y_op);
      st = half_step_ffma_launch(xT, ldx, xsq, xoff, yT, ldy, gc, log_b, nx, ny, d, eps, kappa, fh, workspace, ws_bytes,
                                 s, dyn, 0);
      if (st == TRNOPT_OK)
        st = half_step_ffma_launch(yT, ldy, ysq, yoff, xT, ldx, fh, log_a, ny, nx, d, eps, kappa, gn, workspace,
                                   ws_bytes, s, dyn, 1);
    } else {
      st = TRNOPT_ERR_INVALID_ARGUMENT;
    }
    if (st != TRNOPT_OK) return st;
  }
  return cuda_status(solve_check_launch(static_cast<TrnoptSolveState*>(state), n_iter, g0, g1, w_y, s));
}

int trnopt_max_change(const float* gh_old, const float* gh_new, int n, float inv_eps, float* out, void* stream) {
  if (!gh_old || !gh_new || !out || n < 1) return TRNOPT_ERR_INVALID_ARGUMENT;
  return cuda_status(max_change_launch(gh_old, gh_new, n, inv_eps, out, reinterpret_cast<cudaStream_t>(stream)));
}

static bool plan_args_ok(const double* x, int n, const double* y, int m, int d, double eps) {
  return x && y && n >= 1 && m >= 1 && d >= 1 && eps > 0.0 && isfinite(eps);
}

int trnopt_plan_rows(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                     const double* log_a, const double* log_b, double eps, const int* rows, int nrows, double* out,
                     void* stream) {
  if (!plan_args_ok(x, n, y, m, d, eps) || nrows < 0 || (nrows > 0 && (!rows || !out)))
    return TRNOPT_ERR_INVALID_ARGUMENT;
  if (nrows == 0) return TRNOPT_OK;
  if (!aligned(x, 8) || !aligned(y, 8) || !aligned(out, 8) || !aligned(rows, 4)) return TRNOPT_ERR_ALIGNMENT;
  return cuda_status(plan_rows_launch(x, n, y, m, d, f, g, log_a, log_b, eps, rows, nrows, out,
                                      reinterpret_cast<cudaStream_t>(stream)));
}

size_t trnopt_plan_workspace_size(int n, int m) {
  if (n < 1 || m < 1) return 0;
  return plan_lse_workspace_bytes(current_device(), n, m);
}

int trnopt_plan_log_row_sums(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                             const double* log_a, const double* log_b, double eps, double* out, void* workspace,
                             size_t ws_bytes, void* stream) {
  if (!plan_args_ok(x, n, y, m, d, eps) || !out) return TRNOPT_ERR_INVALID_ARGUMENT;
  const int dev = current_device();
  if (workspace == nullptr || ws_bytes < plan_lse_workspace_bytes(dev, n, m)) return TRNOPT_ERR_WORKSPACE;
  if (!aligned(x, 8) || !aligned(y, 8) || !aligned(out, 8) || !aligned(workspace, 8)) return TRNOPT_ERR_ALIGNMENT;
  return cuda_status(plan_lse_launch(dev, x, n, y, m, d, f, g, log_a, log_b, eps, out, workspace,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
