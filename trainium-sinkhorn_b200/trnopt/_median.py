"""Exact median cost on the GPU for normalization(how="median") (the reference: sinkhorn.py:229-233)."""

from __future__ import annotations

import numpy as np
import torch

from . import _capi


def exact_median_cost(xc: np.ndarray, yc: np.ndarray) -> float:
    """median(max(C, 0)) over all pairs of the centred clouds xc (n, d), yc (m, d), C = |xc_i - yc_j|^2 expanded as
    the reference expands it. The squared norms are summed on the host with numpy, exactly as the reference does;
    the n m costs are evaluated and selected on the current CUDA device without being stored."""
    dev = torch.device("cuda", torch.cuda.current_device())
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a, dtype=np.float64)).to(dev)
    out = _capi.median_cost(t(xc), t(yc), t((xc * xc).sum(1)), t((yc * yc).sum(1)))
    return float(out.item())
