"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for trnopt's log-domain Sinkhorn.

This module is the checker, never the product: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline (the `cpu_baseline` leg and `--impl reference`) may import it. The CUDA product path in
trainium-sinkhorn_b200/ never imports, calls or falls back to it.

It restates the reference's plain-PyTorch CPU solver (evandiewald/trainium-sinkhorn, src/trnopt/sinkhorn.py and
src/trnopt/singlecell.py) in its own code, with the reference's arithmetic order kept wherever it decides the
rounding (the score expression, the max-shifted log-sum-exp, the kappa epilogue), so that in float64 it
reproduces the reference to rounding, and in float32 it is the same CPU workload the reference runs.

Parity of this oracle is pinned against outputs of the reference itself, run in the build container and stored as
fixtures under tests/golden/ by tests/golden/make_golden.py (half-step known answers, the reference test-suite
cases, the 2,000^2 configuration, the normalization scales).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

PAD_LOG_WEIGHT = -1e9     # sinkhorn.py:59 -- log weight of a padding point (finite, so exp() is exactly 0)
DELTA_CAP = 50.0          # sinkhorn.py:60 -- cap on (g_old - g_new) / eps in the balanced marginal check


# --------------------------------------------------------------------------------------------------------------
# The half-step (sinkhorn.py:108-119)
# --------------------------------------------------------------------------------------------------------------

def half_step(x_blk, xsq_blk, off_blk, yT, gh, log_b, inv_eps, eps, kappa):
    """Shifted f update for a block of rows: fh = kappa (|x|^2 + eps off - eps LSE_j z_ij) - |x|^2 with
    z_ij = (2 x_i . y_j + gh_j) / eps + log b_j.  Torch tensors of one dtype; scalars may be 0-d tensors or
    floats.  Follows sinkhorn.py:116-119 term by term (same association, so float64 agrees to rounding)."""
    z = (2.0 * (x_blk @ yT) + gh[None, :]) * inv_eps + log_b[None, :]
    zmax = z.amax(dim=1, keepdim=True)
    lse = zmax[:, 0] + torch.log(torch.exp(z - zmax).sum(dim=1))
    return kappa * (xsq_blk + eps * off_blk - eps * lse) - xsq_blk


def row_lse_np(xa_T: np.ndarray, ya_T: np.ndarray) -> np.ndarray:
    """lse_i = log sum_j exp(xa_i . ya_j) in float64: the quantity of the reference's row-LSE kernel
    (nki_sinkhorn.py:150-172), computed as its known-answer check does (examples/nki_sinkhorn_check.py:33)."""
    s = xa_T.astype(np.float64).T @ ya_T.astype(np.float64)
    mx = s.max(axis=1, keepdims=True)
    return mx[:, 0] + np.log(np.exp(s - mx).sum(axis=1))


# --------------------------------------------------------------------------------------------------------------
# Weights, normalization (sinkhorn.py:211-238)
# --------------------------------------------------------------------------------------------------------------

def log_weights(w, n: int, name: str) -> np.ndarray:
    """sinkhorn.py:211-217: uniform 1/n by default, else log of n positive weights."""
    if w is None:
        return np.full(n, -np.log(n))
    w = np.asarray(w, dtype=np.float64)
    if w.shape != (n,) or np.any(w <= 0):
        raise ValueError(f"{name} must be {n} positive weights")
    return np.log(w)


def normalization(x, y, samples: int = 20_000, seed: int = 0, how: str = "mean"):
    """sinkhorn.py:220-238: centre = mean of both clouds; scale = exact median of all clamped pair costs when
    n m <= 1e8 (how="median"), else the mean (or median) of `samples` random pairs drawn with default_rng(seed)."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    center = np.concatenate([x, y]).mean(axis=0)
    if how == "median" and len(x) * len(y) <= 100_000_000:
        xc, yc = x - center, y - center
        C = ((xc * xc).sum(1)[:, None] + (yc * yc).sum(1)[None, :] - 2.0 * (xc @ yc.T)).ravel()
        scale = float(np.median(np.maximum(C, 0.0)))
        return center, (scale if scale > 0 else 1.0)
    rng = np.random.default_rng(seed)
    i, j = rng.integers(len(x), size=samples), rng.integers(len(y), size=samples)
    dd = ((x[i] - y[j]) ** 2).sum(axis=1)
    scale = float(np.median(dd) if how == "median" else dd.mean())
    return center, (scale if scale > 0 else 1.0)


# --------------------------------------------------------------------------------------------------------------
# The solver (sinkhorn.py:131-394)
# --------------------------------------------------------------------------------------------------------------

@dataclass
class Options:
    """The fields of the reference's SinkhornOptions (sinkhorn.py:63-88) that the CPU solver reads."""
    eps: float = 0.05
    rho: float | tuple | None = None
    max_iters: int = 2000
    tol: float = 1e-4
    check_every: int = 10
    block: int | None = None
    block_y: int | None = None
    eps_start: float | None = None
    eps_decay: float = 0.9
    eps_stages: tuple | None = None
    stage_tol: float = 1e-6
    stage_max_iters: int = 1000
    normalize: bool | str | tuple = True
    fixed_iters: bool = False
    dtype: torch.dtype = torch.float64


@dataclass
class Result:
    f: np.ndarray
    g: np.ndarray
    iterations: int
    error: float
    converged: bool
    cost: float
    seconds: float
    eps: float
    rho: object
    center: np.ndarray
    cost_scale: float
    row_mass: np.ndarray | None = None
    col_mass: np.ndarray | None = None
    stage_iters: list = field(default_factory=list)


class _Side:
    """One cloud, padded to whole blocks (sinkhorn.py:131-157): points, squared norms (float64 then cast), the
    row offsets log(target / reference), log weights (padding: PAD_LOG_WEIGHT) and weights."""

    def __init__(self, pts, log_w, block, dtype, off=None):
        n, d = pts.shape
        nb = -(-n // block)
        P = np.zeros((nb * block, d))
        P[:n] = pts
        L = np.full(nb * block, PAD_LOG_WEIGHT)
        L[:n] = log_w
        O = np.zeros(nb * block)
        if off is not None:
            O[:n] = off
        t = lambda a: torch.as_tensor(np.asarray(a), dtype=dtype)
        self.n, self.block, self.npad = n, block, nb * block
        self.x = t(P)
        self.xT = self.x.T.contiguous()
        self.sq = t((P * P).sum(axis=1))
        self.off, self.zero = t(O), t(np.zeros(nb * block))
        self.log_w, self.w = t(L), t(np.exp(L))


def _sweep(side: _Side, other: _Side, other_h, inv_eps, eps, kappa, use_off=True):
    """One half-step over all row blocks of `side` (sinkhorn.py:170-174)."""
    off = side.off if use_off else side.zero
    parts = []
    for s in range(0, side.npad, side.block):
        e = s + side.block
        parts.append(half_step(side.x[s:e], side.sq[s:e], off[s:e], other.xT, other_h, other.log_w,
                               inv_eps, eps, kappa))
    return torch.cat(parts)


def solve(x, y, a=None, b=None, opts: Options | None = None, a_target=None, b_target=None) -> Result:
    """The reference's sinkhorn() (sinkhorn.py:241-394) on the CPU: validation, normalization, padding, eps
    schedule or stages with the float32 tolerance clamps, the balanced / unbalanced checks, the unshift, the
    unbalanced plan marginals and the cost."""
    opts = opts or Options()
    dt = opts.dtype
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    log_a, log_b = log_weights(a, len(x), "a"), log_weights(b, len(y), "b")
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
    off_x = None if a_target is None else log_weights(a_target, len(x), "a_target") - log_a
    off_y = None if b_target is None else log_weights(b_target, len(y), "b_target") - log_b
    if isinstance(opts.normalize, tuple):
        center, scale = np.asarray(opts.normalize[0], dtype=np.float64), float(opts.normalize[1])
    elif opts.normalize:
        center, scale = normalization(x, y, how=opts.normalize if isinstance(opts.normalize, str) else "mean")
    else:
        center, scale = np.zeros(x.shape[1]), 1.0
    xs, ys = (x - center) / np.sqrt(scale), (y - center) / np.sqrt(scale)
    bx = opts.block or len(x)
    by = opts.block_y or opts.block or len(y)
    X = _Side(xs, log_a, bx, dt, off_x)
    Y = _Side(ys, log_b, by, dt, off_y)

    sched = []
    stages = [e for e in (opts.eps_stages or ()) if e > opts.eps]
    if not stages and opts.eps_start is not None and opts.eps_start > opts.eps:
        e = opts.eps_start
        while e > opts.eps and len(sched) < opts.max_iters:
            sched.append(e)
            e *= opts.eps_decay

    def consts(e, rho):
        kappa = 1.0 if rho is None else rho / (rho + e)
        return tuple(torch.tensor(v, dtype=dt) for v in (1.0 / e, e, kappa))

    gh = torch.zeros(Y.npad, dtype=dt)
    fh = gh
    err, converged, it = float("nan"), False, 0
    stage, stage_it, stage_iters = 0, 0, []
    stage_tol = max(opts.stage_tol, 1e-5 if dt == torch.float32 else 0.0)          # sinkhorn.py:342
    tol = max(opts.tol, 5e-6) if (dt == torch.float32 and not balanced) else opts.tol   # sinkhorn.py:344
    t0 = time.perf_counter()
    while it < opts.max_iters:
        if stages:
            e = stages[stage] if stage < len(stages) else opts.eps
        else:
            e = sched[it] if it < len(sched) else opts.eps
        cx, cy = consts(e, rho_x), consts(e, rho_y)
        inv_eps = cx[0]
        fh = _sweep(X, Y, gh, *cx)
        gh_new = _sweep(Y, X, fh, *cy)
        it += 1
        stage_it += 1
        if stages and stage < len(stages):
            if stage_it % opts.check_every == 0:
                ch = float((((gh_new - gh)[:Y.n].abs().amax()) * inv_eps).item())
                if ch < stage_tol or stage_it >= opts.stage_max_iters:
                    stage_iters.append(stage_it)
                    stage, stage_it = stage + 1, 0
            gh = gh_new
            continue
        check = (not opts.fixed_iters and (stages or it > len(sched))
                 and (stage_it % opts.check_every == 0 or it == opts.max_iters))
        if check:
            if balanced:
                delta = ((gh - gh_new) * inv_eps).clamp(max=DELTA_CAP)
                err = float((Y.w * (torch.exp(delta) - 1.0)).abs().sum().item())
            else:
                err = float((((gh_new - gh)[:Y.n].abs().amax()) * inv_eps).item())
        gh = gh_new
        if check and err < tol:
            converged = True
            break
    if stages:
        stage_iters.append(stage_it)
    f = (fh + X.sq)[:X.n].to(torch.float64).numpy()
    g = (gh + Y.sq)[:Y.n].to(torch.float64).numpy()
    row_mass = col_mass = None
    if not balanced:
        c1 = consts(opts.eps, None)
        fb = (_sweep(X, Y, gh, *c1, use_off=False) + X.sq)[:X.n].to(torch.float64).numpy()
        gb = (_sweep(Y, X, fh, *c1, use_off=False) + Y.sq)[:Y.n].to(torch.float64).numpy()
        row_mass = np.exp(log_a + (f - fb) / opts.eps)
        col_mass = np.exp(log_b + (g - gb) / opts.eps)
    seconds = time.perf_counter() - t0
    cost = float(np.exp(log_a) @ f + np.exp(log_b) @ g) if balanced else float("nan")
    return Result(f=f, g=g, iterations=it, error=err, converged=converged, cost=cost, seconds=seconds,
                  eps=opts.eps, rho=opts.rho, center=center, cost_scale=scale, row_mass=row_mass,
                  col_mass=col_mass, stage_iters=stage_iters)


def transport_plan(x, y, res, a=None, b=None) -> np.ndarray:
    """sinkhorn.py:397-403: the dense plan P_ij = a_i b_j exp((f_i + g_j - C_ij) / eps), float64."""
    x = (np.asarray(x, dtype=np.float64) - res.center) / np.sqrt(res.cost_scale)
    y = (np.asarray(y, dtype=np.float64) - res.center) / np.sqrt(res.cost_scale)
    la, lb = log_weights(a, len(x), "a"), log_weights(b, len(y), "b")
    C = ((x[:, None, :] - y[None, :, :]) ** 2).sum(axis=2)
    return np.exp(la[:, None] + lb[None, :] + (res.f[:, None] + res.g[None, :] - C) / res.eps)


def plan_marginals(x, y, f, g, eps, center, scale, a=None, b=None, chunk: int = 1024):
    """Row and column sums of the plan without holding all of it (float64, chunks of rows)."""
    x = (np.asarray(x, dtype=np.float64) - center) / np.sqrt(scale)
    y = (np.asarray(y, dtype=np.float64) - center) / np.sqrt(scale)
    la, lb = log_weights(a, len(x), "a"), log_weights(b, len(y), "b")
    ysq = (y * y).sum(1)
    rows, cols = np.zeros(len(x)), np.zeros(len(y))
    for s in range(0, len(x), chunk):
        xb = x[s:s + chunk]
        C = (xb * xb).sum(1)[:, None] + ysq[None, :] - 2.0 * (xb @ y.T)
        P = np.exp(la[s:s + chunk, None] + lb[None, :] + (f[s:s + chunk, None] + g[None, :] - C) / eps)
        rows[s:s + chunk] = P.sum(1)
        cols += P.sum(0)
    return rows, cols


def masses_from_potentials(x, y, a, b, f, g, eps: float, chunk: int = 2048):
    """examples/sinkhorn_libs_compare.py:43-56: row and column sums of P = a b^T exp((f + g - C) / eps) on clouds
    that are already normalized, as log-sum-exps over chunks of rows (C expanded as |x|^2 + |y|^2 - 2 x.y)."""
    from scipy.special import logsumexp
    x, y, a, b, f, g = (np.asarray(v, dtype=np.float64) for v in (x, y, a, b, f, g))
    ysq = (y * y).sum(1)
    rows, cols = np.empty(len(x)), np.full(len(y), -np.inf)
    for s in range(0, len(x), chunk):
        xb = x[s:s + chunk]
        C = (xb * xb).sum(1)[:, None] + ysq[None, :] - 2.0 * (xb @ y.T)
        S = (f[s:s + chunk, None] + g[None, :] - C) / eps + np.log(a[s:s + chunk])[:, None] + np.log(b)[None, :]
        rows[s:s + chunk] = np.exp(logsumexp(S, axis=1))
        cols = np.logaddexp(cols, logsumexp(S, axis=0))
    return rows, np.exp(cols)


def pull_back(x0, x1, f, g, eps, center, scale, log_v1, chunk: int = 1024):
    """examples/singlecell_figures.py:35-47: log(P v) over x0 for v = exp(log_v1) over x1, with
    P_ij proportional to exp((f_i + g_j - C_ij) / eps), normalized to log-sum-exp 0."""
    from scipy.special import logsumexp
    s = np.sqrt(float(scale))
    x = (np.asarray(x0, dtype=np.float64) - center) / s
    y = (np.asarray(x1, dtype=np.float64) - center) / s
    f, g, lv = (np.asarray(v, dtype=np.float64) for v in (f, g, log_v1))
    ysq = (y * y).sum(1)
    out = np.empty(len(x))
    for i in range(0, len(x), chunk):
        xb = x[i:i + chunk]
        C = (xb * xb).sum(1)[:, None] + ysq[None, :] - 2.0 * (xb @ y.T)
        out[i:i + chunk] = logsumexp((g[None, :] - C) / eps + lv[None, :], axis=1) + f[i:i + chunk] / eps
    return out - logsumexp(out)


def local_pca_coords(X0, X1, n_components: int = 30, random_state: int = 58951):
    """singlecell.py:30-43: PCA of the centred stacked expression fitted on the transpose, components scaled by the
    singular values. The reference calls scikit-learn's PCA (pinned 1.7.2, uv.lock:3252-3253); this restates the
    algorithm its `auto` policy runs (sklearn/decomposition/_pca.py _fit_full / _fit_truncated,
    sklearn/utils/extmath.py _randomized_svd / _randomized_range_finder / svd_flip) with NumPy and SciPy."""
    from scipy import linalg
    x = np.vstack([np.asarray(X0), np.asarray(X1)]).astype(np.float64)
    x = x - x.mean(axis=0)
    k = min(n_components, x.shape[0])
    A = x.T
    n_samples, n_features = A.shape
    mean = A.mean(axis=0)
    if n_features <= 1000 and n_samples >= 10 * n_features:
        C = A.T @ A - n_samples * np.outer(mean, mean)
        C /= n_samples - 1
        ev, vecs = linalg.eigh(C)
        ev, vecs = ev[::-1].copy(), vecs[:, ::-1].copy()
        ev[ev < 0] = 0.0
        S, Vt = np.sqrt(ev * (n_samples - 1)), vecs.T
    elif max(A.shape) <= 500 or not (1 <= k < 0.8 * min(A.shape)):
        _, S, Vt = linalg.svd(A - mean, full_matrices=False)
    else:
        M = A - mean
        rs = np.random.RandomState(random_state)
        n_random, n_iter = k + 10, (7 if k < 0.1 * min(M.shape) else 4)
        transpose = M.shape[0] < M.shape[1]
        if transpose:
            M = M.T
        Q = rs.normal(size=(M.shape[1], n_random))
        for _ in range(n_iter):
            Q, _ = linalg.lu(M @ Q, permute_l=True)
            Q, _ = linalg.lu(M.T @ Q, permute_l=True)
        Q, _ = linalg.qr(M @ Q, mode="economic")
        Uhat, s, Vb = linalg.svd(Q.T @ M, full_matrices=False)
        U = Q @ Uhat
        S, Vt = (s[:k], U[:, :k].T) if transpose else (s[:k], Vb[:k])
    idx = np.argmax(np.abs(Vt), axis=1)
    Vt = Vt * np.sign(Vt[np.arange(Vt.shape[0]), idx])[:, None]
    comp = Vt[:k].T * S[:k][None, :]
    return comp[:len(X0)], comp[len(X0):]


# --------------------------------------------------------------------------------------------------------------
# wot formulation (singlecell.py:46-86)
# --------------------------------------------------------------------------------------------------------------

def wot_eps_stages(eps: float, eps0: float = 1.0, scalings: int = 5) -> tuple:
    """singlecell.py:46-50: eps0 * sf^-e for e = 0..scalings-1 with sf = eps^(-1/scalings)."""
    sf = np.exp(-np.log(eps) / scalings)
    return tuple(float(eps0 / sf ** e) for e in range(scalings))


def wot_transport_map(x0, x1, growth=None, delta_days=1.0, eps=0.05, lambda1=1.0, lambda2=50.0, growth_iters=1,
                      tol=1e-6, stage_tol=1e-6, opts: Options | None = None):
    """singlecell.py:61-86: median normalization once, rho = (lambda1, lambda2), wot's eps stages, and growth
    iterations that reset the row target to the previous plan's row sums. Returns (result, learned, iters)."""
    from dataclasses import replace
    I, J = len(x0), len(x1)
    G = np.ones(I) if growth is None else np.power(np.asarray(growth, dtype=np.float64), delta_days)
    norm = normalization(x0, x1, how="median")
    base = replace(opts or Options(), eps=eps, rho=(lambda1, lambda2), normalize=norm,
                   eps_stages=wot_eps_stages(eps), stage_tol=stage_tol, tol=tol, eps_start=None, fixed_iters=False)
    a, b = np.full(I, 1.0 / I), np.full(J, 1.0 / J)
    learned, iters, res = [], 0, None
    for i in range(growth_iters):
        if i > 0:
            G = I * res.row_mass
        learned.append(G)
        res = solve(x0, x1, a, b, base, a_target=G / I, b_target=np.full(J, G.mean() / J))
        iters += res.iterations
    return res, learned, iters
