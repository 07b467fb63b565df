"""Entropic optimal transport (log-domain Sinkhorn) with the half-step fused into sm_100a CUDA kernels.

Same API and loop semantics as the reference's src/trnopt/sinkhorn.py (SinkhornOptions, SinkhornResult, sinkhorn,
transport_plan, normalization); the half-step under the loop is this package's C-ABI library instead of the
PyTorch _half_step (sinkhorn.py:108-119) or the NKI kernel (nki_sinkhorn.py:175-228):

    f_i = -eps * LSE_j( log b_j + (g_j - C_ij) / eps )      C_ij = |x_i - y_j|^2
        = |x_i|^2 - eps * LSE_j( log b_j + (gh_j + 2 x_i . y_j) / eps ),   gh = g - |y|^2

computed per row in registers (scores never stored), for all rows of one cloud per launch.

Numerics. The kernels work in float32, like the reference's Trainium and GPU paths. Coordinates are translated so
that the two clouds' joint mean is the origin before they reach the device (C is unchanged by a translation, and
the shifted potentials are re-based so the iteration starts from exactly the reference's g = |y|^2 of its own
frame); this keeps |x|^2 and x.y small and is what the reference's own normalization does when it is on
(sinkhorn.py:224-225). The returned f, g, center and cost_scale are the reference's.

Multi-GPU. With opts.cores = P > 1 the call must be made on every rank of an initialised torch.distributed
process group of P ranks (one GPU each, same inputs): each rank computes 1/P of the rows of every half-step, as the
reference splits rows across NeuronCores and exchanges the halves (sinkhorn.py:295-311). The new potential reaches
every GPU either from the half-step kernel itself, which stores its rows into every GPU's copy over NVLink and
raises an epoch flag that the next half-step waits for (opts.cuda_exchange "peer", the default on the tensor-core
path), or by an NCCL all-gather after each half-step ("nccl").
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _capi
from .backend import Backend

PAD_LOG_WEIGHT = -1e9          # log weight of a padding point (sinkhorn.py:59)
_DELTA_CAP = 50.0              # cap on (g_old - g_new) / eps in the balanced marginal check (sinkhorn.py:60)
ROW_TILE = 128                 # rows per kernel tile: clouds are padded to a multiple of ROW_TILE * shards


@dataclass
class SinkhornOptions:
    eps: float = 0.05
    rho: float | tuple | None = None
    max_iters: int = 2000
    tol: float = 1e-4
    check_every: int = 10
    block: int | None = None       # accepted for compatibility: the fused kernel streams tiles, memory is O(n + m)
    block_y: int | None = None
    eps_start: float | None = None
    eps_decay: float = 0.9
    eps_stages: tuple | None = None
    stage_tol: float = 1e-6
    stage_max_iters: int = 1000
    normalize: bool | str | tuple = True
    fixed_iters: bool = False
    cores: int = 1                 # GPUs (torch.distributed ranks) that split each half-step's rows
    kernel: str = "auto"           # "auto" / "cuda": the fused CUDA half-step (the only one in this package)
    backend: Backend = Backend.preset("cuda-fused")
    cuda_path: str = "auto"        # "tc": tcgen05 split-precision kernel (d <= 64), "ffma": FP32 FFMA tile kernel
    cuda_exchange: str = "auto"    # cores > 1: "peer" (half-steps store their rows into every GPU's copy over
                                   # NVLink; tc path), "nccl" (all-gather after each half-step); auto = peer on tc
                                   #   (any d <= 128), "auto": tc where it applies


@dataclass
class SinkhornResult:
    f: np.ndarray
    g: np.ndarray
    iterations: int
    error: float
    converged: bool
    cost: float
    seconds: float
    eps: float
    rho: float | tuple | None
    center: np.ndarray
    cost_scale: float
    row_mass: np.ndarray | None = None
    col_mass: np.ndarray | None = None
    stage_iters: list = field(default_factory=list)   # eps stages: iterations spent at each stage (the last is the
                                                        # final eps); an addition to the reference's fields


def _use_cuda(opts: SinkhornOptions, d: int) -> None:
    """Kernel selection, the counterpart of the reference's _use_nki (sinkhorn.py:196-208): this package has one
    half-step, so anything but a CUDA float32 backend with kernel "auto" / "cuda" is an error."""
    if opts.kernel not in ("auto", "cuda"):
        raise ValueError(f"kernel={opts.kernel!r}: this package runs only the fused CUDA half-step "
                         "(kernel='cuda' or 'auto')")
    if not opts.backend.is_cuda_fused:
        raise ValueError("the fused CUDA half-step needs a CUDA device and float32: "
                         "use Backend.preset('cuda-fused')")
    if d > 128:
        raise ValueError("the fused CUDA half-step supports d <= 128")
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device: the fused CUDA half-step has no CPU fallback")


def _resolve_path(path: str, d: int) -> str:
    """Which kernel runs the half-step: the tensor-core one on an sm_100 device for d <= 64, else FFMA."""
    if path not in ("auto", "tc", "ffma"):
        raise ValueError(f"cuda_path={path!r}: choose 'auto', 'tc' or 'ffma'")
    tc_ok = _capi.tc_supported(d) and torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10
    if path == "tc" and not tc_ok:
        raise ValueError("cuda_path='tc' needs an sm_100 (B200) device and d <= 64")
    if path == "auto":
        return "tc" if tc_ok else "ffma"
    return path


def _exchange(how: str, path: str) -> str:
    """How the row shards of a half-step reach every GPU: "peer" (stored into every GPU's copy by the kernel that
    computes them; tc path) or "nccl" (an all-gather after the kernel)."""
    if how not in ("auto", "peer", "nccl"):
        raise ValueError(f"cuda_exchange={how!r}: choose 'auto', 'peer' or 'nccl'")
    if how == "peer" and path != "tc":
        raise ValueError("cuda_exchange='peer' needs the tc path")
    if how == "auto":
        return "peer" if path == "tc" else "nccl"
    return how


def _scale_exp(mx: float) -> int:
    """Power-of-two exponent that brings the largest |coordinate| mx into (2^13, 2^14] for the FP16 split of the TC
    path: high enough that the low halves of typical coordinates stay normal FP16 numbers (11 significant bits;
    subnormals keep only absolute precision 2^-24), low enough that hi + lo stays below FP16's 65504."""
    return 0 if mx == 0.0 else 14 - int(np.ceil(np.log2(mx)))


def _log_weights(w, n: int, name: str) -> np.ndarray:
    """sinkhorn.py:211-217."""
    if w is None:
        return np.full(n, -np.log(n))
    w = np.asarray(w, dtype=np.float64)
    if w.shape != (n,) or np.any(w <= 0):
        raise ValueError(f"{name} must be {n} positive weights")
    return np.log(w)


def normalization(x: np.ndarray, y: np.ndarray, samples: int = 20_000, seed: int = 0,
                  how: str = "mean") -> tuple[np.ndarray, float]:
    """(center, cost_scale) as the reference's normalization (sinkhorn.py:220-238): the mean of all points, and the
    mean of `samples` sampled pair costs (how="mean"), or the exact median of all n m clamped costs when
    n m <= 1e8 (how="median", computed on the GPU by a radix select over costs evaluated on the fly in float64;
    larger problems use the median of the sampled pairs). The sampled statistics are computed on the host from
    the same default_rng(seed) draws as the reference."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    center = np.concatenate([x, y]).mean(axis=0)
    return center, _cost_scale(x, y, center, samples, seed, how)


def _cost_scale(x: np.ndarray, y: np.ndarray, center: np.ndarray, samples: int = 20_000, seed: int = 0,
                how: str = "mean") -> float:
    """The second half of normalization (sinkhorn.py:229-238) for a given center: the exact median cost on the GPU
    (how="median", n m <= 1e8), else the mean (or median) of the sampled pair costs (the reference's rng draws)."""
    if how == "median" and len(x) * len(y) <= 100_000_000:
        from ._median import exact_median_cost
        scale = exact_median_cost(x - center, y - center)
        return scale if scale > 0 else 1.0
    rng = np.random.default_rng(seed)
    i, j = rng.integers(len(x), size=samples), rng.integers(len(y), size=samples)
    dd = ((x[i] - y[j]) ** 2).sum(axis=1)
    scale = float(np.median(dd) if how == "median" else dd.mean())
    return scale if scale > 0 else 1.0


class _Cloud:
    """One point cloud on this rank's GPU, padded to a whole number of row tiles per shard.

    xT (d, npad) float32 transposed points (the layout of the reference's NKI path, sinkhorn.py:159-165), sq the
    squared norms (float64, then cast, as sinkhorn.py:149; sq64 keeps the float64 values on the device), log_w
    with PAD_LOG_WEIGHT on padding, w the weights (padding exactly 0), off the row offsets log(target / reference)
    (0 on padding). `pts` is an (n, d) float64 tensor already on the device (or a host array, uploaded here): the
    padding, transpose, norms and weights are all formed on the device."""

    def __init__(self, pts, log_w: np.ndarray, shards: int, dev: torch.device, off=None):
        if not isinstance(pts, torch.Tensor):
            pts = torch.as_tensor(np.ascontiguousarray(pts, dtype=np.float64)).to(dev)
        n, d = pts.shape
        unit = ROW_TILE * shards
        npad = -(-n // unit) * unit
        self.n, self.npad, self.d, self.shards = n, npad, d, shards
        xT = torch.zeros((d, npad), dtype=torch.float32, device=dev)
        xT[:, :n] = pts.T
        self.xT = xT
        vec = torch.zeros((4, npad), dtype=torch.float64, device=dev)
        vec[0, :n] = (pts * pts).sum(dim=1)                  # float64, then cast (sinkhorn.py:149)
        vec[1] = PAD_LOG_WEIGHT
        vec[1, :n] = torch.as_tensor(np.asarray(log_w, dtype=np.float64)).to(dev)
        vec[2] = torch.exp(vec[1])
        if off is not None:
            vec[3, :n] = torch.as_tensor(np.asarray(off, dtype=np.float64)).to(dev)
        self.sq64 = vec[0]
        v32 = vec.to(torch.float32)
        self.sq, self.log_w, self.w, self.off = v32[0], v32[1], v32[2], v32[3]
        self.zero = torch.zeros(npad, dtype=torch.float32, device=dev)
        self.h2d_bytes = 8 * (n * d + n + (n if off is not None else 0))
        self.sexp = _scale_exp(float(pts.abs().max()) if n else 0.0)
        self.packed = None

    def pack(self) -> None:
        """Split the points once into the FP16 [hi | lo] rows of the tensor-core path."""
        if self.packed is None:
            self.packed = _capi.pack_cloud(self.xT, self.npad, self.npad, self.d, self.sexp)
            self.kp = _capi.pack_bytes(1, self.d) // 2


class _DeviceCloud:
    """One cloud in the half-step layout, held in buffers kept between solves of the same shape (_Buffers) and
    filled on the device by trnopt_prepare_cloud: the same attributes as _Cloud (vec = [|x|^2, log w, w, off] as
    float32 rows; sq64 the float64 norms; packed FP16 rows on the tensor-core path, xT on the FFMA path)."""

    def __init__(self, n: int, d: int, shards: int, dev: torch.device, path: str):
        unit = ROW_TILE * shards
        self.n, self.d, self.shards = n, d, shards
        self.npad = npad = -(-n // unit) * unit
        self.pts = torch.empty((n, d), dtype=torch.float64, device=dev)          # upload target
        self.vec = torch.empty((4, npad), dtype=torch.float32, device=dev)
        self.sq, self.log_w, self.w, self.off = self.vec[0], self.vec[1], self.vec[2], self.vec[3]
        self.sq64 = torch.empty(npad, dtype=torch.float64, device=dev)
        self.zero = torch.zeros(npad, dtype=torch.float32, device=dev)
        self.lw_dev = torch.empty(n, dtype=torch.float64, device=dev)            # non-uniform log weights
        self.off_dev = torch.empty(n, dtype=torch.float64, device=dev)
        self.path = path
        if path == "tc":
            self.kp = _capi.pack_bytes(1, d) // 2
            self.packed = torch.empty(npad * self.kp, dtype=torch.float16, device=dev)
            self.xT = None
        else:
            self.packed, self.xT = None, torch.empty((d, npad), dtype=torch.float32, device=dev)
        self.sexp, self.h2d_bytes = 0, 0

    def pack(self) -> None:
        pass

    def upload(self, pts: np.ndarray, log_w: np.ndarray, uniform: bool, off) -> None:
        """Queue the host float64 arrays' copies (asynchronous from page-locked memory)."""
        self.pts.copy_(torch.from_numpy(pts), non_blocking=True)
        self.h2d_bytes = pts.nbytes
        self.uniform = uniform
        if not uniform:
            self.lw_dev.copy_(torch.from_numpy(log_w), non_blocking=True)
            self.h2d_bytes += log_w.nbytes
        self.has_off = off is not None
        if off is not None:
            self.off_dev.copy_(torch.from_numpy(np.ascontiguousarray(off, dtype=np.float64)), non_blocking=True)
            self.h2d_bytes += 8 * self.n

    def prepare(self, center, r, shift, lw_uniform: float, gh0=None) -> None:
        _capi.prepare_cloud(self.pts, self.n, self.npad, center, r, shift, self.sexp,
                            None if self.uniform else self.lw_dev, lw_uniform, self.off_dev if self.has_off else None,
                            self.packed, self.xT, self.vec, self.sq64, gh0)


class _Buffers:
    """Device and page-locked host buffers of one problem shape on one device, kept between calls made from the
    same thread: the uploaded clouds and their layouts, the cloud statistics, the workspace (zeroed once; every
    launch leaves it zeroed), the potentials, and one download buffer for f, g (and the unbalanced masses' half-steps)
    and the device error flags."""

    _cache: dict = {}
    _LIMIT = 4

    @classmethod
    def get(cls, dev, n, m, d, shards, path):
        import threading
        key = (dev.index, n, m, d, shards, path, threading.get_ident())
        b = cls._cache.pop(key, None)
        if b is None:
            b = cls(dev, n, m, d, shards, path)
        cls._cache[key] = b                                 # most recently used last
        while len(cls._cache) > cls._LIMIT:
            cls._cache.pop(next(iter(cls._cache)))
        return b

    @classmethod
    def drop(cls, b) -> None:
        for k, v in list(cls._cache.items()):
            if v is b:
                del cls._cache[k]

    def __init__(self, dev, n, m, d, shards, path):
        self.X = _DeviceCloud(n, d, shards, dev, path)
        self.Y = _DeviceCloud(m, d, shards, dev, path)
        self.stats = torch.empty((2, 3, d), dtype=torch.float64, device=dev)
        self.stats_host = torch.empty((2, 3, d), dtype=torch.float64, pin_memory=True)
        self.stats_scratch = _capi.cloud_stats_scratch(d, dev)
        code = _capi.PATH_TC if path == "tc" else _capi.PATH_FFMA
        need = max(_capi.workspace_size(self.X.npad // shards, self.Y.npad, d, code),
                   _capi.workspace_size(self.Y.npad // shards, self.X.npad, d, code))
        self.ws = _capi.new_workspace(need, dev)
        self.G = [torch.empty(self.Y.npad, dtype=torch.float32, device=dev) for _ in range(2)]
        self.fh = torch.empty(self.X.npad, dtype=torch.float32, device=dev)
        self.hb = torch.empty(max(self.X.npad, self.Y.npad), dtype=torch.float32, device=dev)
        self.out = torch.empty(2 * (n + m) + 1, dtype=torch.float64, device=dev)
        self.out_host = torch.empty(2 * (n + m) + 1, dtype=torch.float64, pin_memory=True)
        self.err = torch.zeros(1, dtype=torch.float32, device=dev)
        self.gauge = torch.zeros(1, dtype=torch.float64, device=dev)     # balanced: offset taken out of g
        self.state = torch.zeros(ctypes.sizeof(_capi.SolveState), dtype=torch.uint8, device=dev)
        self.state_host = torch.zeros(ctypes.sizeof(_capi.SolveState), dtype=torch.uint8, pin_memory=True)

    def read_state(self) -> "_capi.SolveState":
        """The device solve state, copied to the host (synchronises the stream)."""
        self.state_host.copy_(self.state, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return _capi.SolveState.from_buffer_copy(self.state_host.numpy().tobytes())

    def frame(self, center: np.ndarray, r: float) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """After the statistics are on the host: the internal frame's translation (the joint mean of the
        normalised clouds) and each cloud's largest |coordinate| in that frame, with the kernel's arithmetic."""
        st = self.stats_host.numpy()
        n, m = self.X.n, self.Y.n
        shift = ((st[0, 0] - n * center) / r + (st[1, 0] - m * center) / r) / (n + m)
        mx = [max(np.abs((st[c, 2] - center) / r - shift).max(), np.abs((st[c, 1] - center) / r - shift).max())
              for c in (0, 1)]
        return shift, mx[0], mx[1]


class _CudaStep:
    """A half-step with the fused kernel: this rank's share of the rows of `side` against all of `other`, then
    (P > 1) an all-gather so every rank holds the whole new shifted potential. The counterpart of the reference's
    _NkiStep (sinkhorn.py:177-193)."""

    def __init__(self, dev: torch.device, shards: int, rank: int, ws: torch.Tensor, group=None, path: str = "ffma"):
        self.dev, self.shards, self.rank, self.ws, self.group, self.path = dev, shards, rank, ws, group, path

    def rows(self, side: _Cloud) -> tuple[int, int]:
        return _shard_range(side.npad, self.shards, self.rank)

    def __call__(self, side: _Cloud, other: _Cloud, other_h: torch.Tensor, eps: float, kappa: float,
                 use_off: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        out = torch.empty(side.npad, dtype=torch.float32, device=self.dev) if out is None else out
        r0, r1 = self.rows(side)
        off = side.off if use_off else side.zero
        if self.path == "tc":
            _capi.half_step_tc(_Off(side.packed, r0 * side.kp, 2), _Off(side.sq, r0), _Off(off, r0), other.packed,
                               other_h, other.log_w, r1 - r0, other.npad, side.d, side.sexp, other.sexp, eps, kappa,
                               _Off(out, r0), self.ws)
        else:
            _capi.half_step(_Off(side.xT, r0), side.npad, _Off(side.sq, r0), _Off(off, r0), other.xT, other.npad,
                            other_h, other.log_w, r1 - r0, other.npad, side.d, eps, kappa, _Off(out, r0), self.ws)
        if self.shards > 1:
            _gather_rows(out, r0, r1, self.group)
        return out


def _shard_range(npad: int, shards: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of a padded cloud that `rank` computes: equal contiguous shards of whole row tiles."""
    if npad % (ROW_TILE * shards):
        raise ValueError(f"padded size {npad} is not a multiple of {ROW_TILE} * {shards}")
    per = npad // shards
    return rank * per, (rank + 1) * per


def _gather_rows(out: torch.Tensor, r0: int, r1: int, group=None) -> None:
    """In-place all-gather of every rank's rows [r0, r1) of `out` into all of `out` (NCCL on GPUs)."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(out, out[r0:r1], group=group)


class _Off:
    """A device pointer into a tensor at an element offset (for the ctypes calls)."""

    def __init__(self, t: torch.Tensor, offset: int, itemsize: int = 4):
        self.t, self.offset, self.itemsize = t, offset, itemsize

    def data_ptr(self) -> int:
        return self.t.data_ptr() + self.itemsize * self.offset


class _Runs:
    """Runs of n iterations (f then g half-step each) at one (eps, kappa_x, kappa_y). On one GPU a run is queued by a
    single C call (trnopt_sinkhorn_run: the loop body of sinkhorn.py:353-354 issued from C), so the host costs one
    call per run between checks instead of two per iteration. With row shards and a peer region (peer exchange),
    the run is one C call too (trnopt_sinkhorn_run_sharded): each half-step stores its rows into every GPU's copy
    and the GPUs order themselves by epochs. Otherwise (nccl exchange) the run goes half-step by half-step, each
    followed by its NCCL all-gather."""

    def __init__(self, step, X, Y, G, fh, peer=None):
        self.step, self.X, self.Y, self.G, self.fh, self.peer = step, X, Y, G, fh, peer
        self.fused = step.shards == 1

    def sync(self) -> None:
        """Before anything outside the runs reads G or fh: every rank's rows of the last run are in."""
        if self.peer is not None:
            self.peer.wait()

    def run(self, it, n, e, kx, ky):
        X, Y, G, fh, st = self.X, self.Y, self.G, self.fh, self.step
        if self.peer is not None:
            _capi.sinkhorn_run_sharded(self.peer.comm, X.packed, X.sq, X.off, X.log_w, X.npad, X.sexp, Y.packed, Y.sq,
                                       Y.off, Y.log_w, Y.npad, Y.sexp, X.d, G[0], G[1], fh, it % 2, n, e, kx, ky,
                                       st.ws)
            return
        if not self.fused:
            for i in range(it, it + n):
                st(X, Y, G[i % 2], e, kx, out=fh)
                st(Y, X, fh, e, ky, out=G[(i + 1) % 2])
            return
        tc = st.path == "tc"
        _capi.sinkhorn_run(_capi.PATH_TC if tc else _capi.PATH_FFMA,
                           X.packed if tc else X.xT, X.npad, X.sq, X.off, X.log_w, X.npad, X.sexp,
                           Y.packed if tc else Y.xT, Y.npad, Y.sq, Y.off, Y.log_w, Y.npad, Y.sexp, X.d,
                           G[0], G[1], fh, it % 2, n, e, kx, ky, st.ws)


def _prepare_path(path: str, X: _Cloud, Y: _Cloud) -> None:
    if path == "tc":
        X.pack()
        Y.pack()


def _workspace(X: _Cloud, Y: _Cloud, shards: int, dev: torch.device, path: str = "ffma") -> torch.Tensor:
    code = _capi.PATH_TC if path == "tc" else _capi.PATH_FFMA
    need = max(_capi.workspace_size(X.npad // shards, Y.npad, X.d, code),
               _capi.workspace_size(Y.npad // shards, X.npad, X.d, code))
    return _capi.new_workspace(need, dev)


def _device_loop(B, runner, path, opts, stages, sched, balanced, rho_x, rho_y, tol, stage_tol, kap):
    """The loop of sinkhorn.py:346-378 on one GPU with its decisions taken on the device. The eps-scaling prefix
    (eps changes every iteration, no checks) is queued from the host; from there on every run of iterations ends in
    a check kernel that applies the reference loop's rules to a solve state in device memory (trnopt_solve_init /
    trnopt_sinkhorn_run_checked): stage moves, convergence, max_iters. Runs are queued a chunk at a time and the state
    is read once per chunk; runs queued past convergence return at once. The chunk grows from 2 runs with the
    number of runs the last two checks' error ratio predicts are left (at most 16; all of them for fixed_iters).
    Returns (iterations, error, converged, stage iterations)."""
    X, Y, G, fh, ws = runner.X, runner.Y, runner.G, runner.fh, runner.step.ws
    tc = path == "tc"
    it = 0
    for i in range(min(len(sched), opts.max_iters)):
        if balanced:
            _capi.recenter(G[i % 2], Y.n, Y.npad, B.gauge)
        runner.run(i, 1, sched[i], kap(sched[i], rho_x), kap(sched[i], rho_y))
        it = i + 1
    _capi.solve_init(B.state, stages, opts.eps, rho_x, rho_y, opts.check_every, opts.max_iters,
                     opts.stage_max_iters, opts.fixed_iters, len(sched), tol, stage_tol, Y.n, Y.npad, it)
    runs = []
    while it < opts.max_iters:
        n = min(opts.check_every - it % opts.check_every, opts.max_iters - it)
        runs.append((it, n))
        it += n
    chunk, k, prev = (len(runs) if opts.fixed_iters else 2), 0, None
    while k < len(runs):
        for it0, n in runs[k:k + chunk]:
            if balanced:
                _capi.recenter(G[it0 % 2], Y.n, Y.npad, B.gauge, B.state)
            _capi.sinkhorn_run_checked(_capi.PATH_TC if tc else _capi.PATH_FFMA, X.packed if tc else X.xT, X.npad,
                                       X.sq, X.off, X.log_w, X.npad, X.sexp, Y.packed if tc else Y.xT, Y.npad, Y.sq,
                                       Y.off, Y.log_w, Y.npad, Y.sexp, X.d, G[0], G[1], fh, it0 % 2, n, B.state,
                                       Y.w, ws)
        k += chunk
        st = B.read_state()
        if st.done:
            break
        chunk = 16
        e = float(st.err)
        if prev is not None and np.isfinite(e) and 0.0 < e < prev[0] and prev[0] > 0.0:
            rate = (e / prev[0]) ** (1.0 / max(1, k - prev[1]))
            if 0.0 < rate < 1.0 and e > tol:
                chunk = int(min(16, max(1, np.ceil(np.log(tol / e) / np.log(rate)))))
        if np.isfinite(e):
            prev = (e, k)
    st = B.read_state()
    stage_iters = list(st.stage_iters[:st.stage]) + ([st.stage_it] if stages else [])
    return int(st.it), float(st.err), bool(st.converged), stage_iters


def sinkhorn(x, y, a=None, b=None, opts: SinkhornOptions | None = None, a_target=None,
             b_target=None) -> SinkhornResult:
    """Entropic OT between point clouds x (n, d) and y (m, d) with weights a, b (default uniform): the reference's
    sinkhorn() (sinkhorn.py:241-394) with the half-steps on the GPU.

    a, b are the reference measure of the entropy term, eps KL(P | a b^T). Unbalanced (rho given), the penalties
    rho KL(P 1 | a_target) and rho KL(P^T 1 | b_target) pull the plan's marginals toward a_target and b_target
    (default a and b)."""
    opts = opts or SinkhornOptions()
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    log_a, log_b = _log_weights(a, len(x), "a"), _log_weights(b, len(y), "b")
    balanced = opts.rho is None
    if balanced and abs(np.exp(log_a).sum() - np.exp(log_b).sum()) > 1e-9 * np.exp(log_a).sum():
        raise ValueError("balanced OT needs sum(a) == sum(b); pass rho for unbalanced")
    if balanced and (a_target is not None or b_target is not None):
        raise ValueError("a_target / b_target are for unbalanced OT (pass rho)")
    if balanced:
        rho_x = rho_y = None
    elif isinstance(opts.rho, (tuple, list)):
        rho_x, rho_y = opts.rho
    else:
        rho_x = rho_y = opts.rho
    off_x = None if a_target is None else _log_weights(a_target, len(x), "a_target") - log_a
    off_y = None if b_target is None else _log_weights(b_target, len(y), "b_target") - log_b
    _use_cuda(opts, x.shape[1])
    shards = max(1, int(opts.cores))
    rank, group = 0, None
    if shards > 1:
        import torch.distributed as dist
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() != shards:
            raise ValueError(f"cores={shards} needs an initialised torch.distributed group of {shards} ranks "
                             "(one GPU per rank, launched with torchrun)")
        rank = dist.get_rank()
    dev = opts.backend.torch_device()

    norm_how = None
    if isinstance(opts.normalize, tuple):
        center, scale = np.asarray(opts.normalize[0], dtype=np.float64), float(opts.normalize[1])
    elif opts.normalize:
        # normalization(x, y, how): the center (the mean of all points) comes from the device's per-coordinate sums
        # below, so the host makes no pass over the points (at 262,144^2 the host concatenate-and-mean took ~0.1 s)
        norm_how = opts.normalize if isinstance(opts.normalize, str) else "mean"
        center, scale = None, None
    else:
        center, scale = np.zeros(x.shape[1]), 1.0

    with torch.cuda.device(dev):
        # One float64 upload per cloud into buffers kept for this shape; the per-coordinate statistics on the device
        # (one small download and the call's one mid-way synchronisation) give the internal frame (the normalised
        # clouds' joint mean at the origin) and the FP16 split scales; then each cloud's layout (the reference's
        # _Cloud, sinkhorn.py:131-167, after the normalisation of :268-269) is written by one kernel.
        path = _resolve_path(opts.cuda_path, x.shape[1])
        B = _Buffers.get(dev, len(x), len(y), x.shape[1], shards, path)
        X, Y = B.X, B.Y
        ua, ub = a is None, b is None
        X.upload(np.ascontiguousarray(x), log_a, ua, off_x)
        Y.upload(np.ascontiguousarray(y), log_b, ub, off_y)
        _capi.cloud_stats(X.pts, Y.pts, B.stats, B.stats_scratch)
        B.stats_host.copy_(B.stats, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        if norm_how is not None:
            st = B.stats_host.numpy()
            center = (st[0, 0] + st[1, 0]) / (len(x) + len(y))
            scale = _cost_scale(x, y, center, how=norm_how)
        r = float(np.sqrt(scale))
        center = np.asarray(center, dtype=np.float64)
        shift, mx, my = B.frame(center, r)
        X.sexp, Y.sexp = _scale_exp(mx), _scale_exp(my)
        step = _CudaStep(dev, shards, rank, B.ws, group, path)

        sched = []
        stages = [e for e in (opts.eps_stages or ()) if e > opts.eps]
        if not stages and opts.eps_start is not None and opts.eps_start > opts.eps:
            e = opts.eps_start
            while e > opts.eps and len(sched) < opts.max_iters:
                sched.append(e)
                e *= opts.eps_decay

        def kap(e, rho):
            return 1.0 if rho is None else rho / (rho + e)

        # Ping-pong potentials: before iteration i the shifted g is G[i % 2]; fh has one buffer. The reference starts
        # from gh = 0 in its frame, i.e. g = |ys|^2; in the internal frame that is gh = |ys|^2 - |yi|^2 (exactly the
        # same iteration), written into G[0] by Y's layout kernel.
        peer = None
        if shards > 1 and _exchange(opts.cuda_exchange, path) == "peer":
            from . import _comm
            peer = _comm.region(4 * (X.npad + 2 * Y.npad), group)
            fh = peer.tensor(0, X.npad)
            G = [peer.tensor(4 * X.npad, Y.npad), peer.tensor(4 * (X.npad + Y.npad), Y.npad)]
        else:
            G, fh = B.G, B.fh
        X.prepare(center, r, shift, log_a[0])
        Y.prepare(center, r, shift, log_b[0], gh0=G[0])
        fh.zero_()
        B.gauge.zero_()
        if peer is not None:
            peer.arrive()                                  # the others may write into these buffers from here on
        err_dev = B.err
        runner = _Runs(step, X, Y, G, fh, peer)
        err, converged, it = float("nan"), False, 0
        stage, stage_it, stage_iters = 0, 0, []
        stage_tol = max(opts.stage_tol, 1e-5)              # float32 floors (sinkhorn.py:342-344)
        tol = max(opts.tol, 5e-6) if not balanced else opts.tol
        t0 = time.perf_counter()
        if shards == 1:
            it, err, converged, stage_iters = _device_loop(B, runner, path, opts, stages, sched, balanced, rho_x,
                                                           rho_y, tol, stage_tol, kap)
        while shards > 1 and it < opts.max_iters:
            # The loop of sinkhorn.py:346-378, advanced a run of iterations at a time: a run ends where the host
            # has to look (a check, an eps change, max_iters), so the iterations inside it are one C call.
            if stages:
                e = stages[stage] if stage < len(stages) else opts.eps
            else:
                e = sched[it] if it < len(sched) else opts.eps
            if not stages and it < len(sched):
                n = 1                                          # eps-scaling schedule: eps changes every iteration
            else:
                n = opts.check_every - (stage_it % opts.check_every)
            n = min(n, opts.max_iters - it)
            if balanced:
                # the run's input potential moved to mean zero, the offset kept in float64 (trnopt_recenter)
                _capi.recenter(G[it % 2], Y.n, Y.npad, B.gauge)
            runner.run(it, n, e, kap(e, rho_x), kap(e, rho_y))
            runner.sync()
            it += n
            stage_it += n
            gh_prev, gh_new = G[(it - 1) % 2], G[it % 2]
            inv_eps = float(np.float32(1.0 / e))
            if stages and stage < len(stages):
                if stage_it % opts.check_every == 0:
                    _capi.max_change(gh_prev, gh_new, Y.n, inv_eps, err_dev)
                    ch = float(err_dev.item())
                    if ch < stage_tol or stage_it >= opts.stage_max_iters:
                        stage_iters.append(stage_it)
                        stage, stage_it = stage + 1, 0
                continue
            check = (not opts.fixed_iters and (stages or it > len(sched))
                     and (stage_it % opts.check_every == 0 or it == opts.max_iters))
            if check:
                if balanced:
                    _capi.balanced_error(gh_prev, gh_new, Y.w, Y.npad, inv_eps, err_dev)
                else:
                    _capi.max_change(gh_prev, gh_new, Y.n, inv_eps, err_dev)
                err = float(err_dev.item())
            if check and err < tol:
                converged = True
                break
        if stages and shards > 1:
            stage_iters.append(stage_it)
        gh = G[it % 2]
        # Unshift on the device into one float64 buffer (f, g, and for unbalanced the balanced half-steps' fb, gb),
        # the error flags at its end, one download (sinkhorn.py:375-389).
        nx, ny = X.n, Y.n
        out = B.out
        gauge = B.gauge if balanced else None
        _capi.unshift(fh, X.sq64, nx, out, gauge, -1)
        _capi.unshift(gh, Y.sq64, ny, _Off(out, nx, 8), gauge, 1)
        if not balanced:
            # The plan's marginals from one balanced (kappa = 1, no offset) update each way (sinkhorn.py:381-389).
            hx = step(X, Y, gh, opts.eps, 1.0, use_off=False, out=B.hb[:X.npad])
            _capi.unshift(hx, X.sq64, nx, _Off(out, nx + ny, 8))
            hy = step(Y, X, fh, opts.eps, 1.0, use_off=False, out=B.hb[:Y.npad])
            _capi.unshift(hy, Y.sq64, ny, _Off(out, 2 * nx + ny, 8))
        total = 2 * (nx + ny) + 1
        _capi.take_error_flags(_Off(out, total - 1, 8))
        B.out_host[:total].copy_(out[:total], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        host = B.out_host.numpy()
        flags = int(host[total - 1])
        if flags:
            _Buffers.drop(B)                                # its workspace may hold a stopped launch's counters
            raise _capi.TrnoptError(f"a kernel reported device error flags {flags:#x} during the solve")
        f, g = host[:nx].copy(), host[nx:nx + ny].copy()
        row_mass = col_mass = None
        if not balanced:
            fb, gb = host[nx + ny:2 * nx + ny], host[2 * nx + ny:2 * (nx + ny)]
            row_mass = np.exp(log_a + (f - fb) / opts.eps)
            col_mass = np.exp(log_b + (g - gb) / opts.eps)
        seconds = time.perf_counter() - t0
    cost = float(np.exp(log_a) @ f + np.exp(log_b) @ g) if balanced else float("nan")
    return SinkhornResult(f=f, g=g, iterations=it, error=err, converged=converged, cost=cost, seconds=seconds,
                          eps=opts.eps, rho=opts.rho, center=center, cost_scale=scale, row_mass=row_mass,
                          col_mass=col_mass, stage_iters=stage_iters)


def transport_plan(x, y, res: SinkhornResult, a=None, b=None) -> np.ndarray:
    """The dense plan P (n x m, float64) from a result: for small problems and tests only (sinkhorn.py:397-403).
    Evaluated in float64 by the library's plan kernel (trnopt.plan)."""
    from .plan import transport_plan as _plan
    return _plan(x, y, res, a, b)
