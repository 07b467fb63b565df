"""The transport plan evaluated from a solve's potentials on the GPU, in float64, never stored whole.

For a result res of sinkhorn(x, y, a, b, ...) the plan is
    P_ij = a_i b_j exp((f_i + g_j - C_ij) / eps),   C_ij = |x_i - y_j|^2 on (x - center) / sqrt(cost_scale),
the plan of the reference's transport_plan (sinkhorn.py:397-403). The reference evaluates it, and the quantities
built from it, on the host with NumPy in float64; here the same float64 arithmetic runs in the library's plan kernels
(trnopt_plan_rows, trnopt_plan_log_row_sums):

    transport_plan(x, y, res, a, b)           dense P (small problems), as the reference
    plan_rows(x, y, res, rows, a, b)          selected rows of P
    plan_marginals(x, y, res, a, b)           row and column sums of P
    masses_from_potentials(x, y, a, b, f, g, eps)
                                              the same sums on already-normalized clouds
                                              (examples/sinkhorn_libs_compare.py:43-56)
    pull_back(x0, x1, res, log_v1)            normalized log(P v), the ancestor pull-back
                                              (examples/singlecell_figures.py:35-47)

The sums are float64 log-sum-exps, so rows whose terms all underflow exp() still come out right in log form.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _capi


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("trnopt.plan needs a CUDA device (the plan kernels have no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def _dev(a, dev, dtype=torch.float64):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a, dtype=np.float64)).to(dev, dtype)


def _log_w(w, n: int, name: str) -> np.ndarray:
    """sinkhorn.py:211-217: log of the given weights, or log(1/n)."""
    if w is None:
        return np.full(n, -np.log(n))
    w = np.asarray(w, dtype=np.float64)
    if w.shape != (n,) or np.any(w <= 0):
        raise ValueError(f"{name} must be {n} positive weights")
    return np.log(w)


def _normalized(x, y, res):
    """(x - center) / sqrt(cost_scale) in float64 on the host, as sinkhorn.py:399-400."""
    s = np.sqrt(res.cost_scale)
    x = (np.asarray(x, dtype=np.float64) - res.center) / s
    y = (np.asarray(y, dtype=np.float64) - res.center) / s
    if x.ndim != 2 or y.ndim != 2 or x.shape[1] != y.shape[1]:
        raise ValueError("x (n, d) and y (m, d) must share d")
    return x, y


def _inputs(x, y, res, a, b):
    dev = _device()
    x, y = _normalized(x, y, res)
    if np.shape(res.f) != (len(x),) or np.shape(res.g) != (len(y),):
        raise ValueError("the result's potentials do not match x and y")
    la, lb = _log_w(a, len(x), "a"), _log_w(b, len(y), "b")
    return dev, _dev(x, dev), _dev(y, dev), _dev(res.f, dev), _dev(res.g, dev), _dev(la, dev), _dev(lb, dev)


def plan_rows(x, y, res, rows, a=None, b=None) -> np.ndarray:
    """Rows P[rows, :] (len(rows), m) in float64. Row indices follow NumPy rules (negative counts from the end)."""
    n = len(x)
    idx = np.asarray(rows, dtype=np.int64).reshape(-1)
    if np.any(idx < -n) or np.any(idx >= n):
        raise IndexError(f"row index out of range for {n} rows")
    idx = np.where(idx < 0, idx + n, idx).astype(np.int32)
    dev, xd, yd, f, g, la, lb = _inputs(x, y, res, a, b)
    out = _capi.plan_rows(xd, yd, f, g, la, lb, res.eps, torch.as_tensor(idx).to(dev))
    return out.cpu().numpy()


def transport_plan(x, y, res, a=None, b=None) -> np.ndarray:
    """The dense plan P (n x m, float64) from a result (sinkhorn.py:397-403): small problems and tests."""
    return plan_rows(x, y, res, np.arange(len(x)), a, b)


def plan_marginals(x, y, res, a=None, b=None) -> tuple[np.ndarray, np.ndarray]:
    """(P 1, P^T 1): the plan's row and column sums in float64."""
    dev, xd, yd, f, g, la, lb = _inputs(x, y, res, a, b)
    rows = _capi.plan_log_row_sums(xd, yd, f, g, la, lb, res.eps)
    cols = _capi.plan_log_row_sums(yd, xd, g, f, lb, la, res.eps)
    return torch.exp(rows).cpu().numpy(), torch.exp(cols).cpu().numpy()


def masses_from_potentials(x, y, a, b, f, g, eps: float) -> tuple[np.ndarray, np.ndarray]:
    """Row and column sums of P = a b^T exp((f + g - C) / eps) for clouds x, y that are already normalized
    (examples/sinkhorn_libs_compare.py:43-56, whose eps is its module constant)."""
    dev = _device()
    x, y = np.asarray(x, dtype=np.float64), np.asarray(y, dtype=np.float64)
    xd, yd = _dev(x, dev), _dev(y, dev)
    f, g = _dev(f, dev), _dev(g, dev)
    la = _dev(np.log(np.asarray(a, dtype=np.float64)), dev)
    lb = _dev(np.log(np.asarray(b, dtype=np.float64)), dev)
    rows = _capi.plan_log_row_sums(xd, yd, f, g, la, lb, eps)
    cols = _capi.plan_log_row_sums(yd, xd, g, f, lb, la, eps)
    return torch.exp(rows).cpu().numpy(), torch.exp(cols).cpu().numpy()


def pull_back(x0, x1, res, log_v1) -> np.ndarray:
    """The ancestor pull-back through one transport map (examples/singlecell_figures.py:35-47): with
    P_ij ∝ exp((f_i + g_j - C_ij) / eps) and a distribution v over x1 given as log_v1, returns log(P v)
    normalized to log-sum-exp 0 over x0."""
    dev = _device()
    x, y = _normalized(x0, x1, res)
    lv = np.asarray(log_v1, dtype=np.float64)
    if lv.shape != (len(y),):
        raise ValueError(f"log_v1 must have shape ({len(y)},)")
    out = _capi.plan_log_row_sums(_dev(x, dev), _dev(y, dev), _dev(res.f, dev), _dev(res.g, dev), None,
                                  _dev(lv, dev), res.eps)
    return (out - torch.logsumexp(out, 0)).cpu().numpy()
