"""Seeded synthetic point clouds for the five benchmark configurations of this build.

The reference measures on a real single-cell dataset (Schiebinger et al. reprogramming data) that is not
available here; configs 3 and 4 are seeded synthetic stand-ins with the same shapes (the largest day pair,
7,355 x 8,962 cells in a 30-d local PCA, and a 38-pair / 175k-cell trajectory). Configs 1, 2 and 5 are fully
synthetic in the reference's own benchmark too (examples/sinkhorn_benchmark.py:13-16, the FlashSinkhorn
10k x 10k setup).

Every generator is deterministic in numpy's PCG64 (`np.random.default_rng`), so the same arrays come out on any
machine with the same numpy major version.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def cfg1(seed: int = 0):
    """Balanced, n = m = 2,000, d = 16, x, y ~ U[0, 1]^16 (the correctness configuration)."""
    rng = np.random.default_rng(seed)
    return rng.uniform(size=(2000, 16)), rng.uniform(size=(2000, 16))


def cfg2(seed: int = 0, n: int = 10_000, m: int | None = None, d: int = 64):
    """Balanced, n = m = 10,000, d = 64, x, y ~ U[0, 1]^64 (the headline single-GPU configuration)."""
    rng = np.random.default_rng(seed)
    return rng.uniform(size=(n, d)), rng.uniform(size=(m or n, d))


def _mixture_centres(rng, k: int, d: int):
    return rng.normal(scale=2.0, size=(k, d))                       # centres ~ N(0, 4 I)


def _mixture_points(rng, centres, weights, n: int):
    k, d = centres.shape
    lab = rng.choice(k, size=n, p=weights)
    sd = 1.0 / np.sqrt(np.arange(1, d + 1))                          # variance 1/k along axis k (PCA-like decay)
    return centres[lab] + rng.normal(size=(n, d)) * sd[None, :]


def cfg3(seed: int = 3, n: int = 7355, m: int = 8962, d: int = 30, k: int = 25):
    """Unbalanced single-cell-shaped pair: 25-component Gaussian mixture in d = 30, targets shifted by a random
    drift of norm 1, growth weights G ~ exp(N(0, 0.5^2)). Returns (x0, x1, growth)."""
    rng = np.random.default_rng(seed)
    centres = _mixture_centres(rng, k, d)
    w = np.full(k, 1.0 / k)
    x0 = _mixture_points(rng, centres, w, n)
    drift = rng.normal(size=d)
    drift /= np.linalg.norm(drift)
    x1 = _mixture_points(rng, centres + drift[None, :], w, m)
    growth = np.exp(rng.normal(scale=0.5, size=n))
    return x0, x1, growth


@dataclass
class Trajectory:
    cohorts: list            # per time point: (n_t, 30) coordinates
    growth: list             # per time point: (n_t,) growth weights


def cfg4(seed: int = 4, n_times: int = 39, total: int = 175_000, d: int = 30, k: int = 25) -> Trajectory:
    """39 cohorts (38 consecutive pairs) of total ~175k cells, sizes U[1000, 9000] rescaled to the total;
    mixture weights and centres drift linearly in time."""
    rng = np.random.default_rng(seed)
    sizes = rng.uniform(1000, 9000, size=n_times)
    sizes = np.maximum(1, np.round(sizes * total / sizes.sum())).astype(int)
    c0 = _mixture_centres(rng, k, d)
    c1 = c0 + rng.normal(scale=1.0, size=(k, d))                     # where the centres end up
    w0, w1 = rng.dirichlet(np.ones(k)), rng.dirichlet(np.ones(k))
    cohorts, growth = [], []
    for t in range(n_times):
        s = t / max(1, n_times - 1)
        w = (1 - s) * w0 + s * w1
        cohorts.append(_mixture_points(rng, (1 - s) * c0 + s * c1, w / w.sum(), int(sizes[t])))
        growth.append(np.exp(rng.normal(scale=0.5, size=int(sizes[t]))))
    return Trajectory(cohorts=cohorts, growth=growth)


def cfg5(seed: int = 5, n: int = 262_144, m: int | None = None, d: int = 64):
    """Large balanced problem: x, y ~ N(0, I_64) / 8, n = m = 262,144."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=(n, d), dtype=np.float32) / 8.0
    y = rng.standard_normal(size=(m or n, d), dtype=np.float32) / 8.0
    return x.astype(np.float64), y.astype(np.float64)


def cfg5_eps_stages(eps_start: float = 1.0, eps_end: float = 0.01, stages: int = 8) -> tuple:
    """Geometric eps stages from eps_start down to eps_end over `stages` values; the intermediate ones (all but
    the last) go to SinkhornOptions.eps_stages, the last is SinkhornOptions.eps."""
    e = np.geomspace(eps_start, eps_end, stages)
    return tuple(float(v) for v in e[:-1])


# Test shapes for local_pca_coords, one per solver sklearn's PCA picks: (cells0, cells1, genes, seed).
PCA_CASES = {"randomized": (300, 400, 1200, 11), "randomized_t": (500, 400, 600, 12), "full": (80, 100, 300, 13),
             "covariance_eigh": (50, 70, 2400, 14)}


def expression(cells0: int, cells1: int, genes: int, seed: int = 0, factors: int = 12):
    """Seeded synthetic expression for two time points (cells x genes, float64): log1p of Poisson counts whose rates
    come from a low-rank model (cell-state factors drifting between the time points times gene loadings), the shape
    of the wot inputs to local_pca_coords (a stand-in for the reprogramming data, which is absent)."""
    rng = np.random.default_rng(seed)
    load = rng.gamma(0.6, 1.0, size=(factors, genes))
    base = rng.normal(-1.0, 0.6, size=genes)

    def cells(n, shift):
        z = rng.normal(0.0, 1.0, size=(n, factors)) * 0.5 + shift
        rate = np.exp(np.clip(base[None, :] + 0.4 * z @ load / np.sqrt(factors), -8, 6))
        return np.log1p(rng.poisson(rate)).astype(np.float64)

    drift = rng.normal(0.0, 0.3, size=factors)
    return cells(cells0, 0.0), cells(cells1, drift)
