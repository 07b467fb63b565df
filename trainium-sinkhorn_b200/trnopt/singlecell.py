"""Waddington-OT-style transport maps between consecutive time points, on the fused CUDA Sinkhorn.

The same functions and formulation as the reference's src/trnopt/singlecell.py (wot, Schiebinger et al. 2019):
cost = squared distance / its exact median (computed once per pair, on the GPU), uniform reference measure,
row target = growth G / I, column target = mean(G) / J, KL penalties (lambda1, lambda2), wot's eps stages, and
growth iterations that set the next row target to the previous plan's row sums.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, replace

import numpy as np

from .sinkhorn import SinkhornOptions, SinkhornResult, normalization, sinkhorn, transport_plan


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
