"""Waddington-OT-style transport maps between consecutive time points, on the fused CUDA Sinkhorn.

The same functions and formulation as the reference's src/trnopt/singlecell.py (wot, Schiebinger et al. 2019):
cost = squared distance / its exact median (computed once per pair, on the GPU), uniform reference measure,
row target = growth G / I, column target = mean(G) / J, KL penalties (lambda1, lambda2), wot's eps stages, and
growth iterations that set the next row target to the previous plan's row sums. `wot_trajectory` runs the maps of
every consecutive pair of a time course (the loop of the reference's examples/singlecell_wot.py) and can write each
pair's potentials in that example's npz layout and restart from them (`save_pair`, `load_pair`).
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, replace
from pathlib import Path

import numpy as np
import torch

from .sinkhorn import SinkhornOptions, SinkhornResult, normalization, sinkhorn, transport_plan


PCA_RANDOM_STATE = 58951      # singlecell.py:42 (wot.ot.compute_pca's seed)


def local_pca_coords(X0, X1, n_components: int = 30) -> tuple[np.ndarray, np.ndarray]:
    """wot's per-pair embedding (singlecell.py:30-43): PCA of the two time points' expression together, fitted on
    the transpose (genes as samples, cells as features) after centring each gene, as wot.ot.compute_pca does with
    sklearn's PCA(n_components, random_state=58951); the cells' coordinates are the components scaled by the
    singular values. Returns (cells0 x k, cells1 x k) in float64.

    The arithmetic runs on the current CUDA device in float64 and follows the solver sklearn's PCA picks for the
    shape (its `auto` policy): `randomized` for the usual sizes (the same Gaussian test matrix, drawn on the host
    from RandomState(58951), LU-normalised power iterations, economic QR, thin SVD, sign flip on the rows of Vt),
    `full` for small problems, `covariance_eigh` for few cells and many genes."""
    import scipy.sparse as sp
    if not torch.cuda.is_available():
        raise RuntimeError("local_pca_coords needs a CUDA device (no CPU path in this package)")
    dev = torch.device("cuda", torch.cuda.current_device())
    m1 = X0.toarray() if sp.issparse(X0) else np.asarray(X0)
    m2 = X1.toarray() if sp.issparse(X1) else np.asarray(X1)
    n0 = len(m1)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a, dtype=np.float64)).to(dev)
    x = torch.cat([t(m1), t(m2)])                      # cells x genes
    x = x - x.mean(dim=0)
    k = min(n_components, x.shape[0])
    A = x.T                                            # sklearn's X: genes (samples) x cells (features)
    n_samples, n_features = A.shape
    if n_features <= 1000 and n_samples >= 10 * n_features:
        solver = "covariance_eigh"
    elif max(A.shape) <= 500:
        solver = "full"
    elif 1 <= k < 0.8 * min(A.shape):
        solver = "randomized"
    else:
        solver = "full"
    mean = A.mean(dim=0)
    if solver == "full":
        _, S, Vt = torch.linalg.svd(A - mean, full_matrices=False)
    elif solver == "covariance_eigh":
        C = A.T @ A - n_samples * torch.outer(mean, mean)
        C = C / (n_samples - 1)
        ev, vecs = torch.linalg.eigh(C)
        ev, vecs = torch.flip(ev, dims=[0]), torch.flip(vecs, dims=[1])
        ev = torch.clamp(ev, min=0.0)
        S, Vt = torch.sqrt(ev * (n_samples - 1)), vecs.T
    else:
        S, Vt = _randomized_svd(A - mean, k, np.random.RandomState(PCA_RANDOM_STATE), dev)
    Vt = _flip_rows(Vt)
    comp = (Vt[:k].T * S[:k][None, :]).cpu().numpy()
    return comp[:n0], comp[n0:]


def _randomized_svd(M: torch.Tensor, k: int, rs: np.random.RandomState, dev, n_oversamples: int = 10):
    """Halko et al.'s randomized SVD as sklearn.utils.extmath._randomized_svd runs it for PCA (n_iter 'auto',
    LU normaliser, transpose 'auto', no sign flip inside): returns (s[:k], Vt[:k]) of M."""
    n_random = k + n_oversamples
    n_iter = 7 if k < 0.1 * min(M.shape) else 4
    transpose = M.shape[0] < M.shape[1]
    if transpose:
        M = M.T
    Q = torch.as_tensor(rs.normal(size=(M.shape[1], n_random))).to(dev)
    def lu_pl(a):
        P, L, _ = torch.linalg.lu(a)
        return P @ L
    norm = lu_pl if n_iter > 2 else (lambda a: a)
    for _ in range(n_iter):
        Q = norm(M @ Q)
        Q = norm(M.T @ Q)
    Q, _ = torch.linalg.qr(M @ Q, mode="reduced")
    Uhat, s, Vt = torch.linalg.svd(Q.T @ M, full_matrices=False)
    U = Q @ Uhat
    if transpose:
        return s[:k], U[:, :k].T
    return s[:k], Vt[:k]


def _flip_rows(Vt: torch.Tensor) -> torch.Tensor:
    """sklearn's svd_flip(u_based_decision=False): each row's largest-|.| entry made positive."""
    idx = torch.argmax(Vt.abs(), dim=1)
    signs = torch.sign(Vt[torch.arange(Vt.shape[0], device=Vt.device), idx])
    return Vt * signs[:, None]


def wot_eps_stages(eps: float, eps0: float = 1.0, scalings: int = 5) -> tuple:
    """Intermediate eps values of wot's duality-gap solver: eps0 * sf^-e for e = 0 .. scalings - 1 with
    sf = eps^(-1 / scalings) (singlecell.py:46-50)."""
    sf = np.exp(-np.log(eps) / scalings)
    return tuple(float(eps0 / sf ** e) for e in range(scalings))


@dataclass
class TransportMap:
    result: SinkhornResult
    learned_growth: list
    seconds: float
    iterations: int


def wot_transport_map(x0: np.ndarray, x1: np.ndarray, growth: np.ndarray | None = None, delta_days: float = 1.0,
                      eps: float = 0.05, lambda1: float = 1.0, lambda2: float = 50.0, growth_iters: int = 1,
                      tol: float = 1e-6, stage_tol: float = 1e-6, opts: SinkhornOptions | None = None) -> TransportMap:
    """One wot transport map between coordinates x0 (I cells at t0) and x1 (J cells at t1) (singlecell.py:61-86).
    opts supplies backend, cores, check_every and max_iters; eps, rho, normalize and the stages are set here."""
    I, J = len(x0), len(x1)
    G = np.ones(I) if growth is None else np.power(np.asarray(growth, dtype=np.float64), delta_days)
    t = time.perf_counter()
    norm = normalization(x0, x1, how="median")
    seconds = time.perf_counter() - t
    base = replace(opts or SinkhornOptions(), eps=eps, rho=(lambda1, lambda2), normalize=norm,
                   eps_stages=wot_eps_stages(eps), stage_tol=stage_tol, tol=tol, eps_start=None, fixed_iters=False)
    a, b = np.full(I, 1.0 / I), np.full(J, 1.0 / J)
    learned, iters, res = [], 0, None
    for i in range(growth_iters):
        if i > 0:
            G = I * res.row_mass
        learned.append(G)
        t = time.perf_counter()
        res = sinkhorn(x0, x1, a, b, base, a_target=G / I, b_target=np.full(J, G.mean() / J))
        seconds += time.perf_counter() - t
        iters += res.iterations
    return TransportMap(result=res, learned_growth=learned, seconds=seconds, iterations=iters)


def wot_tmap(x0, x1, tm: TransportMap) -> np.ndarray:
    """The dense transport map in wot's normalization (I * P), on the host; small pairs only (singlecell.py:89-92)."""
    I, J = len(x0), len(x1)
    return I * transport_plan(x0, x1, tm.result, np.full(I, 1.0 / I), np.full(J, 1.0 / J))


# The keys of the reference example's per-pair files (examples/singlecell_wot.py:112-117).
PAIR_KEYS = ("f", "g", "eps", "center", "cost_scale", "row_mass", "col_mass", "learned_growth", "cells0", "cells1",
             "x0", "x1")


@dataclass
class SavedPair:
    tm: TransportMap
    x0: np.ndarray
    x1: np.ndarray
    cells0: np.ndarray
    cells1: np.ndarray


def pair_path(directory, t0: float, t1: float) -> Path:
    """directory / pair_{t0:g}_{t1:g}.npz, the reference example's file name (examples/singlecell_wot.py:114)."""
    return Path(directory) / f"pair_{t0:g}_{t1:g}.npz"


def save_pair(path, tm: TransportMap, x0, x1, cells0=None, cells1=None) -> Path:
    """Write one pair's potentials, masses and learned growth under the reference example's keys (PAIR_KEYS), plus
    `iterations`, `seconds`, `rho`, `error` and `converged`. Cell names are stored as unicode arrays (no pickled
    objects; None stores the row indices). The file appears whole or not at all (written beside it, then renamed),
    so a pipeline killed mid-write leaves nothing that a restart would half-read."""
    r = tm.result
    x0, x1 = np.asarray(x0, dtype=np.float64), np.asarray(x1, dtype=np.float64)
    c0 = np.arange(len(x0)).astype(str) if cells0 is None else np.asarray(cells0, dtype=str)
    c1 = np.arange(len(x1)).astype(str) if cells1 is None else np.asarray(cells1, dtype=str)
    none = np.zeros(0)
    arrays = dict(f=r.f, g=r.g, eps=r.eps, center=r.center, cost_scale=r.cost_scale,
                  row_mass=none if r.row_mass is None else r.row_mass,
                  col_mass=none if r.col_mass is None else r.col_mass,
                  learned_growth=np.array(tm.learned_growth), cells0=c0, cells1=c1, x0=x0, x1=x1,
                  iterations=tm.iterations, seconds=tm.seconds,
                  rho=np.array(np.nan if r.rho is None else r.rho, dtype=np.float64), error=r.error,
                  converged=r.converged)
    path = Path(path)
    tmp = path.with_name(path.name + ".partial")
    with open(tmp, "wb") as fh:
        np.savez(fh, **arrays)
    os.replace(tmp, path)
    return path


def load_pair(path, allow_pickle: bool = False) -> SavedPair:
    """Read a file of save_pair or of the reference example. The reference stores cell names as object arrays, which
    NumPy loads only with allow_pickle=True (pickles run code: pass it only for files you trust). Keys the reference
    does not write come back as: iterations 0, seconds 0, rho None, error NaN, converged False."""
    with np.load(path, allow_pickle=allow_pickle) as z:
        missing = [k for k in PAIR_KEYS if k not in z.files]
        if missing:
            raise ValueError(f"{path}: not a pair file (missing {', '.join(missing)})")
        d = {k: z[k] for k in z.files}
    rho = None
    if "rho" in d and not np.all(np.isnan(d["rho"])):
        rho = tuple(float(v) for v in np.atleast_1d(d["rho"]))
        rho = rho[0] if len(rho) == 1 else rho
    mass = lambda v: None if v.size == 0 else v                  # noqa: E731
    res = SinkhornResult(f=d["f"], g=d["g"], iterations=int(d.get("iterations", 0)), error=float(d.get("error", np.nan)),
                         converged=bool(d.get("converged", False)), cost=float("nan"),
                         seconds=float(d.get("seconds", 0.0)), eps=float(d["eps"]), rho=rho, center=d["center"],
                         cost_scale=float(d["cost_scale"]), row_mass=mass(d["row_mass"]), col_mass=mass(d["col_mass"]))
    tm = TransportMap(result=res, learned_growth=list(np.atleast_2d(d["learned_growth"])),
                      seconds=float(d.get("seconds", 0.0)), iterations=int(d.get("iterations", 0)))
    return SavedPair(tm=tm, x0=d["x0"], x1=d["x1"], cells0=d["cells0"], cells1=d["cells1"])


def wot_trajectory(cohorts, times=None, growth=None, *, n_components: int | None = None, save=None,
                   resume: bool = False, cells=None, **map_kwargs) -> list:
    """Transport maps for every consecutive pair of a time course: the loop of the reference's
    examples/singlecell_wot.py:79-117. cohorts[k] is the (cells, features) matrix at times[k] (default 0, 1, ...).
    Per pair (t0, t1): with n_components, both cohorts are embedded by local_pca_coords (as the example does with
    expression), else their rows are the coordinates; the growth rates growth[k] are raised to t1 - t0; one
    wot_transport_map (map_kwargs: eps, lambda1, lambda2, growth_iters, tol, stage_tol, opts). With save=DIR each
    pair is written to pair_path(DIR, t0, t1) (save_pair, cell names from cells[k] if given); with resume=True a pair
    whose file exists is loaded instead of solved, so an interrupted run restarts at its first missing pair. A file
    written for other coordinates raises ValueError. Returns the TransportMaps in pair order."""
    times = list(range(len(cohorts))) if times is None else [float(t) for t in times]
    if len(times) != len(cohorts):
        raise ValueError(f"{len(cohorts)} cohorts but {len(times)} times")
    if growth is not None and len(growth) < len(cohorts) - 1:
        raise ValueError("growth needs one vector per cohort (the last is not used)")
    if resume and save is None:
        raise ValueError("resume=True needs save=DIR")
    if save is not None:
        Path(save).mkdir(parents=True, exist_ok=True)
    maps = []
    for k in range(len(cohorts) - 1):
        t0, t1 = times[k], times[k + 1]
        if n_components:
            x0, x1 = local_pca_coords(cohorts[k], cohorts[k + 1], n_components)
        else:
            x0, x1 = np.asarray(cohorts[k], dtype=np.float64), np.asarray(cohorts[k + 1], dtype=np.float64)
        path = None if save is None else pair_path(save, t0, t1)
        if resume and path.exists():
            sp = load_pair(path)
            if sp.x0.shape != x0.shape or sp.x1.shape != x1.shape or not (
                    np.array_equal(sp.x0, x0) and np.array_equal(sp.x1, x1)):
                raise ValueError(f"{path} was written for other coordinates: remove it or pass resume=False")
            maps.append(sp.tm)
            continue
        tm = wot_transport_map(x0, x1, None if growth is None else growth[k], t1 - t0, **map_kwargs)
        if path is not None:
            save_pair(path, tm, x0, x1, None if cells is None else cells[k], None if cells is None else cells[k + 1])
        maps.append(tm)
    return maps
