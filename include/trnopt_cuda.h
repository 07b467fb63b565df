/* trnopt_cuda.h -- C ABI of the B200 (sm_100a) fused log-domain Sinkhorn half-step library (libtrnopt_cuda.so).
 *
 * This library replaces the hot path of trnopt (evandiewald/trainium-sinkhorn): the half-step
 *     fh_i = kappa * (|x_i|^2 + eps * off_i - eps * lse_i) - |x_i|^2,
 *     lse_i = log sum_j exp( (2 x_i . y_j + gh_j) / eps + log b_j )
 * of src/trnopt/sinkhorn.py:108-119 (the PyTorch _half_step) and src/trnopt/nki_sinkhorn.py:175-228 (the fused
 * NKI kernel), plus the companions around it in the solver loop.
 *
 * Conventions
 *   - Plain pointers and sizes only. Every array pointer is a DEVICE pointer on the calling thread's current CUDA
 *     device; `stream` is a cudaStream_t (NULL = the legacy default stream). Calls are asynchronous on `stream`
 *     unless stated otherwise.
 *   - Point clouds are passed transposed, as the reference's kernel takes them (xa_T / yT in
 *     nki_sinkhorn.py:175-182): xT[k * ldx + i] is coordinate k of point i. ldx >= rows, ldx % 4 == 0, and xT,
 *     yT are 16-byte aligned. All floating-point arrays are float32.
 *   - Every entry point returns TRNOPT_OK (0) or a negative status; trnopt_status_string() names it. Nothing
 *     is launched when an argument check fails.
 *   - The caller owns all memory. The library never allocates device memory on these paths and never frees
 *     caller memory. Scratch space is a caller-provided workspace (see trnopt_workspace_size).
 */
#ifndef TRNOPT_CUDA_H_
#define TRNOPT_CUDA_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TRNOPT_OK = 0,
  TRNOPT_ERR_INVALID_ARGUMENT = -1, /* a size, scalar or null pointer is out of range */
  TRNOPT_ERR_ALIGNMENT = -2,        /* a pointer or leading dimension breaks the alignment rules above */
  TRNOPT_ERR_WORKSPACE = -3,        /* workspace missing or smaller than trnopt_workspace_size() */
  TRNOPT_ERR_UNSUPPORTED = -4,      /* shape or path not supported on this build / device */
  TRNOPT_ERR_CUDA = -5,             /* a CUDA runtime call failed (trnopt_last_cuda_error() has the code) */
  TRNOPT_ERR_DEVICE = -6,           /* a kernel reported an error flag (see trnopt_device_error_flags) */
  TRNOPT_ERR_TOO_LARGE = -7         /* needs more scratch than the library's static array (no-allocation entry) */
};

enum { TRNOPT_PATH_FFMA = 0, TRNOPT_PATH_TC = 1 };

/* Library version, e.g. 100 for 0.1.0. No reference counterpart. */
int trnopt_version(void);

/* Human-readable name of a status code. */
const char* trnopt_status_string(int status);

/* The cudaError_t of the last failed CUDA call made by this library on the calling thread (0 if none). */
int trnopt_last_cuda_error(void);

/* Synchronises `stream`, then reads and clears the device error word of the current device: bit 1 = a bounded
 * wait inside a kernel gave up, bit 2 = tensor-memory allocation gave up, bit 4 = a launch invariant failed,
 * bit 8 = another GPU of a sharded run did not publish its rows in time.
 * The reference has no device-side errors; its failures are Python exceptions (sinkhorn.py:201-207). */
int trnopt_device_error_flags(void* stream, int* flags_out);

/* Bytes of workspace that trnopt_half_step / trnopt_row_lse (path FFMA) or trnopt_half_step_tc (path TC) need
 * for `rows` x `m` on the current device. The workspace holds per-row partial (max, sum) pairs of split rows and
 * one arrival counter per 128-row tile. Replaces the reference's per-call intermediates (the dense score tile
 * of sinkhorn.py:116, the on-chip per-chunk statistics of nki_sinkhorn.py:87-96). */
size_t trnopt_workspace_size(int rows, int m, int d, int path);

/* Zero a workspace once after allocating it. The kernels leave it zeroed again when they finish, so one init
 * serves any number of calls on one stream; calls that overlap on the GPU must use separate workspaces. */
int trnopt_workspace_init(void* workspace, size_t ws_bytes, void* stream);

/* The fused half-step, FP32 FFMA tile path. Replaces _half_step (sinkhorn.py:108-119) and the NKI kernel
 * make_half_step_kernel(d, rows, m)(xa_T, xsq, off, yT, gh, log_b, sc) (nki_sinkhorn.py:175-228):
 *   xT (d, ldx)  rows of this side, transposed        xsq (rows,)  |x_i|^2
 *   off (rows,)  log(target / reference) or NULL (= 0) yT (d, ldy)  the other side, transposed
 *   gh (m,)      shifted potential of the other side    log_b (m,)   log weights of the other side
 *   eps, kappa   the scalars of sc = [2/eps, 1/eps, eps, kappa] (sinkhorn.py:331-333)
 *   fh (rows,)   output: the new shifted potential
 * 1 <= d <= 128. Padding columns carry log_b = -1e9 exactly as in the reference (sinkhorn.py:59,144). */
int trnopt_half_step(const float* xT, int ldx, const float* xsq, const float* off, const float* yT, int ldy,
                     const float* gh, const float* log_b, int rows, int m, int d, float eps, float kappa,
                     float* fh, void* workspace, size_t ws_bytes, void* stream);

/* Tensor-core path. A cloud is split once per solve into FP16 pairs, x 2^scale_exp = hi + lo, stored as n rows of
 * [hi (dk) | lo (dk) | zeros] (dk = d rounded up to 16; trnopt_pack_bytes gives the size; 128-byte aligned).
 * scale_exp is chosen by the caller so that max |x| 2^scale_exp lies in (2^13, 2^14] (hi + lo below FP16's
 * 65504, low halves of typical coordinates normal FP16 numbers). The counterpart
 * of the reference's once-per-solve kernel layout, the [x ; 1] blocks of _Cloud (sinkhorn.py:159-165).
 * Supported for d <= 64. */
size_t trnopt_pack_bytes(int n, int d);
int trnopt_pack_cloud(const float* xT, int ldx, int n, int d, int scale_exp, void* packed, void* stream);

/* The fused half-step on tcgen05 tensor cores (same contract as trnopt_half_step, sinkhorn.py:108-119 /
 * nki_sinkhorn.py:175-228): x . y as xh.yh + xh.yl + xl.yh in FP16 with FP32 accumulation (about 22 significant
 * bits), the bias gh / eps + log b added in the accumulator by one more MMA of its three-part BF16 split (24
 * significant bits), online row log-sum-exp. xpack = rows packed rows of this side
 * (scale sx), ypack = m packed rows of the other side (scale sy). Needs an sm_100 device; workspace from
 * trnopt_workspace_size(rows, m, d, TRNOPT_PATH_TC). */
int trnopt_half_step_tc(const void* xpack, const float* xsq, const float* off, const void* ypack, const float* gh,
                        const float* log_b, int rows, int m, int d, int sx, int sy, float eps, float kappa, float* fh,
                        void* workspace, size_t ws_bytes, void* stream);

/* The tensor-core half-step without a workspace argument, for callers that cannot allocate device memory (code
 * inside someone else's stream capture, plugin hosts that only pass in/out buffers, arena allocators sized at
 * start-up). No counterpart in the reference. Same arguments and results as trnopt_half_step_tc; the scratch is a
 * static device array of trnopt_static_scratch_bytes() (4 MiB) per GPU, held until the process exits. Problems
 * that need more (trnopt_workspace_size(rows, m, d, TRNOPT_PATH_TC) > 4 MiB) return TRNOPT_ERR_TOO_LARGE without
 * launching. The first call on a GPU looks up the array's device address (cudaGetSymbolAddress) with that GPU
 * current: make it before any stream capture. All calls on a GPU share the array: calls whose kernels overlap on
 * the GPU (several streams or threads) race and give wrong results. Allocates nothing. */
size_t trnopt_static_scratch_bytes(void);
int trnopt_half_step_tc_static(const void* xpack, const float* xsq, const float* off, const void* ypack,
                               const float* gh, const float* log_b, int rows, int m, int d, int sx, int sy, float eps,
                               float kappa, float* fh, void* stream);

/* Row log-sum-exp of a product, lse_i = log sum_j exp(xa_i . ya_j), xa_T (k, ldx), ya_T (k, ldy), 1 <= k <= 128.
 * Replaces make_row_lse_kernel(K, rows, m)(xa_T, ya_T) (nki_sinkhorn.py:150-172). */
int trnopt_row_lse(const float* xaT, int ldx, const float* yaT, int ldy, int rows, int m, int k, float* lse,
                   void* workspace, size_t ws_bytes, void* stream);

/* Convergence checks of the solver loop (sinkhorn.py:358-374), reduced on the device into out[0]:
 *   balanced:   sum_j | w_j (exp(min((gh_old_j - gh_new_j) * inv_eps, 50)) - 1) |   (sinkhorn.py:370-371)
 *   max change: max_j |gh_new_j - gh_old_j| * inv_eps over j < n                    (sinkhorn.py:360, 373) */
int trnopt_balanced_error(const float* gh_old, const float* gh_new, const float* w, int n, float inv_eps,
                          float* out, void* stream);
int trnopt_max_change(const float* gh_old, const float* gh_new, int n, float inv_eps, float* out, void* stream);

/* Balanced solves only: move the potential gh (npad entries, the first n real) by K = its mean over the n real
 * entries rounded to float32, gh -= K, and add K to gauge[0] (float64, device). The plan and, in exact arithmetic,
 * the iteration are unchanged by a constant c in (f + c, g - c) (the balanced problem's gauge freedom, which the
 * reference's loop carries from its start g = |y|^2); keeping the stored potentials near zero keeps float32's
 * absolute precision on them. The caller puts the offset back (trnopt_unshift with sign +1 for g, -1 for f).
 * state: NULL, or a TrnoptSolveState (below) whose done flag makes the call return at once.
 * No reference counterpart (the reference's float64 path does not need it). */
int trnopt_recenter(float* gh, int n, int npad, double* gauge, const void* state, void* stream);

/* n_iter Sinkhorn iterations in one call: for i < n_iter, with g = (start_parity + i) odd ? g1 : g0 and the other
 * buffer g',  fh <- half_step(x side, y side, g, kappa_x);  g' <- half_step(y side, x side, fh, kappa_y),
 * i.e. the body of the reference's loop, sweep(Xs, Ys, ...) then sweep(Ys, Xs, ...) (sinkhorn.py:353-354),
 * queued from C so a run of iterations between host checks costs one call. path TRNOPT_PATH_TC takes packed clouds
 * (x_op, y_op from trnopt_pack_cloud, scales sx, sy; ldx, ldy unused); TRNOPT_PATH_FFMA takes transposed clouds
 * (x_op = xT (d, ldx), y_op = yT (d, ldy)). nx, ny are the (padded) point counts, log_a / log_b the log weights,
 * xoff / yoff the row offsets (or NULL). One workspace sized for the larger of the two half-steps. */
int trnopt_sinkhorn_run(int path, const void* x_op, int ldx, const float* xsq, const float* xoff, const float* log_a,
                        int nx, int sx, const void* y_op, int ldy, const float* ysq, const float* yoff,
                        const float* log_b, int ny, int sy, int d, float* g0, float* g1, float* fh, int start_parity,
                        int n_iter, float eps, float kappa_x, float kappa_y, void* workspace, size_t ws_bytes,
                        void* stream);

/* Solve set-up and tear-down on the device, after one float64 upload per cloud. Replace the host work of the
 * reference's sinkhorn() around the loop: normalisation arithmetic (sinkhorn.py:268-269), the _Cloud layout
 * (sinkhorn.py:131-167: padding, squared norms in float64 then cast, PAD_LOG_WEIGHT log weights, weights, row
 * offsets) and the unshift of the returned potentials (sinkhorn.py:375-376).
 *
 * trnopt_cloud_stats: stats (2, 3, d) float64 = for cloud 0 (x, n rows) and cloud 1 (y, m rows) of row-major
 *   (count, d) float64 points, the per-coordinate sum, min and max. Fixed partition and reduction order (the same
 *   result on every run). scratch: trnopt_cloud_stats_scratch_bytes(d) bytes, 256-byte aligned, zeroed once; left
 *   zeroed. d <= 128.
 * trnopt_prepare_cloud: for point i < n, with u = (pts_i - center) / r and v = u - shift (float64; center and
 *   shift are HOST arrays of d doubles, read during the call): sq64[i] = |v|^2, vec (4, npad) float32 rows
 *   [|v|^2, log w_i, w_i, off_i], packed row i = the FP16 [hi | lo] split of v 2^scale_exp (as trnopt_pack_cloud;
 *   if packed != NULL), xT[k * npad + i] = v_k (if xT != NULL), gh0[i] = |u|^2 - |v|^2 (if gh0 != NULL: the
 *   reference's starting g = |y|^2 in the shifted frame). log_w NULL = log_w_uniform for every point; off NULL = 0.
 *   Rows n <= i < npad are padding: zeros, log w = -1e9, w = 0.
 * trnopt_unshift: out[i] = (h[i] + sq[i]) + sign * gauge[0] in float64, i < n (f = fh + |x|^2, with the offset
 *   that trnopt_recenter took out of a balanced solve's potentials put back; gauge NULL = 0; sign +1 or -1).
 * trnopt_take_error_flags: out[0] = the device error word (as trnopt_device_error_flags reports it), which is
 *   cleared; asynchronous, so one download can bring potentials and flags back together. */
size_t trnopt_cloud_stats_scratch_bytes(int d);
int trnopt_cloud_stats(const double* x, int n, const double* y, int m, int d, double* stats, void* scratch,
                       size_t scratch_bytes, void* stream);
int trnopt_prepare_cloud(const double* pts, int n, int d, int npad, const double* center, double r,
                         const double* shift, int scale_exp, const double* log_w, double log_w_uniform,
                         const double* off, void* packed, float* xT, float* vec, double* sq64, float* gh0,
                         void* stream);
int trnopt_unshift(const float* h, const double* sq, int n, const double* gauge, int sign, double* out,
                   void* stream);
int trnopt_take_error_flags(double* out, void* stream);

/* The solver loop decided on the GPU. The reference's loop (sinkhorn.py:346-378) looks at the potentials every
 * check_every iterations on the host: the balanced marginal error or the maximum potential change, a move to the
 * next eps stage, convergence. Here that state lives in device memory and a check kernel applies the same rules
 * after each run of iterations, so the host can queue many runs and read the state once:
 *   trnopt_solve_init          fill a TrnoptSolveState (device memory, sizeof(TrnoptSolveState) bytes, 8-byte
 *                              aligned) with the plan and the loop's starting counters (it0: iterations already run,
 *                              e.g. an eps-scaling prefix; the stage counter starts equal to it). Synchronous copy.
 *   trnopt_sinkhorn_run_checked
 *                              trnopt_sinkhorn_run with eps and the kappas of the state's current stage, then the
 *                              check for the run's end (n_iter must end at a check point: it0 + iterations run so
 *                              far + n_iter a multiple of check_every, or max_iters). w_y: the y side's weights
 *                              (npad entries, 0 on padding) for the balanced error. Once the state is done
 *                              (converged, or max_iters reached) every later half-step, check and recentring
 *                              returns at once, leaving the potentials of the converged iteration in place.
 * The fields below `it` are the loop's counters and result (read them from a copy of the struct on the host):
 * it = iterations, converged, err = the last check's value, stage_iters[k] = iterations spent at intermediate stage
 * k (k < stage). No reference counterpart as an interface: it restates the reference loop's decisions. */
#define TRNOPT_MAX_STAGES 32
typedef struct TrnoptSolveState {
  double stage_eps[TRNOPT_MAX_STAGES + 1]; /* intermediate eps values, then the final eps at [n_stages] */
  double rho[2];                           /* marginal penalties of the x and y sides; < 0: balanced (kappa 1) */
  float tol, stage_tol;                    /* as the reference clamps them for float32 (sinkhorn.py:342-344) */
  int n_stages, check_every, max_iters, stage_max_iters, fixed_iters, balanced, sched_len, n_real, npad;
  float eps, kappa[2], dot2, gh2;          /* the current stage's half-step parameters (float, as a host call) */
  int it, stage, stage_it, done, converged;
  float err;
  int stage_iters[TRNOPT_MAX_STAGES + 1];
} TrnoptSolveState;
int trnopt_solve_init(void* state, const double* stage_eps, int n_stages, double final_eps, double rho_x,
                      double rho_y, int check_every, int max_iters, int stage_max_iters, int fixed_iters,
                      int sched_len, float tol, float stage_tol, int n_real, int npad, int it0, void* stream);
int trnopt_sinkhorn_run_checked(int path, const void* x_op, int ldx, const float* xsq, const float* xoff,
                                const float* log_a, int nx, int sx, const void* y_op, int ldy, const float* ysq,
                                const float* yoff, const float* log_b, int ny, int sy, int d, float* g0, float* g1,
                                float* fh, int start_parity, int n_iter, void* state, const float* w_y,
                                void* workspace, size_t ws_bytes, void* stream);

/* Self-test of the FMA-pipe 2^x used to balance exps between MUFU and the FMA units (no reference counterpart):
 * out[i] = 2^x[i] for n floats, max relative error 2.1e-7 over [-125, 100]. */
int trnopt_test_ex2_poly(const float* x, float* out, int n, void* stream);

/* Exact median of all n m clamped costs max(C_ij, 0), C_ij = (sqx_i + sqy_j) - 2 xc_i . yc_j, float64, written to
 * out[0]; the mean of the two middle values when n m is even (np.median). xc (n, d) and yc (m, d) are row-major
 * centred points, sqx / sqy their squared norms. n m <= 1e8, d <= 128. Replaces the host NumPy median of
 * normalization(how="median") (sinkhorn.py:229-233). The costs are re-evaluated in 16 passes and never stored;
 * the workspace (trnopt_median_workspace_size bytes, 256-byte aligned) needs no initialisation. */
size_t trnopt_median_workspace_size(void);
int trnopt_median_cost(const double* xc, const double* yc, const double* sqx, const double* sqy, int n, int m, int d,
                       double* out, void* workspace, size_t ws_bytes, void* stream);

/* Multi-GPU (one process per GPU, up to 8): a peer-mapped region per rank and a sharded run that publishes each
 * half-step's rows straight into every GPU's copy of the potential over NVLink. Replaces the reference's
 * cross-core exchange after each half-step (sinkhorn.py:295-311: blocks split over cores, then concatenated on
 * the host) and the all-gather a per-half-step design would need.
 *
 *   trnopt_comm_create    allocate this rank's region (bytes for the caller's buffers, after a 256-byte flag
 *                         header) on the current device and write its IPC handle (trnopt_comm_handle_bytes bytes)
 *                         to handle_out. Blocking.
 *   trnopt_comm_open      map every other rank's region from the world handles (rank order, concatenated), which
 *                         the caller exchanges through its process group. Blocking.
 *   trnopt_comm_buffer    this rank's buffers (the same offset names the same vector on every rank).
 *   trnopt_comm_arrive    queue a signal to every rank that this rank's stream has reached this point (call it
 *                         after initialising the buffers of a solve, before its first run).
 *   trnopt_comm_wait      queue a wait until every other rank has published everything this rank has published
 *                         so far; call before reading a gathered vector outside the run (checks, downloads).
 *   trnopt_sinkhorn_run_sharded
 *                         trnopt_sinkhorn_run (TRNOPT_PATH_TC) over row shards: rank r computes rows
 *                         [r nx / W, (r + 1) nx / W) of each f half-step and the same share of each g half-step
 *                         and publishes them; g0, g1 and fh must lie in the comm buffer; nx, ny multiples of 128 W.
 *   trnopt_comm_destroy   unmap the peers and free the region. Every rank must be past its last access to the
 *                         others' regions (synchronise, then a host barrier) before any rank destroys.
 * Every rank makes the same sequence of arrive / run / wait calls. All waits are bounded (4 s): an expired wait
 * sets error flag 8 (trnopt_device_error_flags). Epochs, not the calls, order the GPUs: no host synchronisation
 * is needed between runs. */
size_t trnopt_comm_handle_bytes(void);
int trnopt_comm_create(int rank, int world, size_t bytes, void** comm_out, void* handle_out);
int trnopt_comm_open(void* comm, const void* handles);
void* trnopt_comm_buffer(void* comm);
size_t trnopt_comm_buffer_bytes(void* comm);
unsigned long long trnopt_comm_epoch(void* comm);
int trnopt_comm_arrive(void* comm, void* stream);
int trnopt_comm_wait(void* comm, void* stream);
int trnopt_comm_destroy(void* comm);
int trnopt_sinkhorn_run_sharded(void* comm, const void* xpack, const float* xsq, const float* xoff,
                                const float* log_a, int nx, int sx, const void* ypack, const float* ysq,
                                const float* yoff, const float* log_b, int ny, int sy, int d, float* g0, float* g1,
                                float* fh, int start_parity, int n_iter, float eps, float kappa_x, float kappa_y,
                                void* workspace, size_t ws_bytes, void* stream);

/* Plan evaluation from potentials, float64, for P_ij = exp(log_a_i + log_b_j + (f_i + g_j - C_ij) / eps) with the
 * direct-difference cost C_ij = sum_k (x_ik - y_jk)^2. x (n, d) and y (m, d) are row-major, already centred and
 * scaled as the solve saw them ((x - center) / sqrt(cost_scale)); f, g, log_a, log_b may each be NULL (= 0).
 *
 * trnopt_plan_rows: out (nrows, m) row-major = the rows P[rows[r], :]; rows (device int array) must lie in [0, n)
 * (a row index outside gives a row of NaN, nothing out of bounds is read). Replaces the dense host evaluation of
 * transport_plan (sinkhorn.py:397-403) and wot_tmap (singlecell.py:89-92) for the rows asked for.
 *
 * trnopt_plan_log_row_sums: out (n,) = log sum_j P_ij (-inf where the row is all zero), computed as a float64
 * log-sum-exp; deterministic. Swapping (x, n, f, log_a) with (y, m, g, log_b) gives log column sums. Replaces the
 * host loops of masses_from_potentials (examples/sinkhorn_libs_compare.py:43-56) and, with log_a = NULL and
 * log_b = log v, the ancestor pull-back log(P v) (examples/singlecell_figures.py:35-47, before its final
 * normalisation). Needs a workspace of trnopt_plan_workspace_size(n, m) bytes (8-byte aligned, no
 * initialisation); one workspace per stream. */
int trnopt_plan_rows(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                     const double* log_a, const double* log_b, double eps, const int* rows, int nrows, double* out,
                     void* stream);
size_t trnopt_plan_workspace_size(int n, int m);
int trnopt_plan_log_row_sums(const double* x, int n, const double* y, int m, int d, const double* f, const double* g,
                             const double* log_a, const double* log_b, double eps, double* out, void* workspace,
                             size_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRNOPT_CUDA_H_ */
