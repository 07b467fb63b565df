"""The no-allocation entry point (trnopt_half_step_tc_static) against the workspace entry point.

Callers that cannot allocate device memory -- code running inside a stream capture they do not own, plugin hosts
that only hand over input and output buffers, arena allocators fixed at start-up -- use the variant whose scratch is
a static array inside the library. This file is collected last so that a run stopping at its first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import numpy as np
import pytest
import torch

from trnopt import _capi

pytestmark = pytest.mark.gpu
HS_TOL = 5e-5          # |delta fh| / eps, the half-step tolerance of the other GPU tests


def _dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32).cuda()


def _problem(rows, m, d, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(rows, d)) / np.sqrt(2 * d)
    y = rng.normal(size=(m, d)) / np.sqrt(2 * d)
    gh = -(y * y).sum(1) + rng.normal(scale=0.2, size=m)
    lb = np.full(m, -np.log(m))
    return x, y, gh, lb, rng.normal(scale=0.3, size=rows)


def _scale(a):
    return 14 - int(np.ceil(np.log2(np.abs(a).max())))


def test_static_scratch_matches_workspace_entry_on_two_calls():
    rows, m, d, eps, kappa = 3000, 7000, 64, 0.1, 0.9
    assert _capi.workspace_size(rows, m, d, _capi.PATH_TC) <= _capi.lib.trnopt_static_scratch_bytes()
    x, y, gh, lb, off = _problem(rows, m, d, 11)
    xT, ldx = _capi._pad_ld(_dev(x.T))
    yT, ldy = _capi._pad_ld(_dev(y.T))
    sx, sy = _scale(x), _scale(y)
    xp, yp = _capi.pack_cloud(xT, ldx, rows, d, sx), _capi.pack_cloud(yT, ldy, m, d, sy)
    args = (_dev((x * x).sum(1)), _dev(off), yp, _dev(gh), _dev(lb), rows, m, d, sx, sy, eps, kappa)
    ref = torch.empty(rows, device="cuda")
    ws = _capi.new_workspace(_capi.workspace_size(rows, m, d, _capi.PATH_TC), "cuda")
    _capi.half_step_tc(xp, *args, ref, ws)
    for _ in range(2):                                   # the second call reuses what the first left behind
        out = torch.full((rows,), float("nan"), device="cuda")
        _capi.half_step_tc_static(xp, *args, out)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item() / eps
        assert np.isfinite(out.cpu().numpy()).all() and err <= HS_TOL, err
    assert _capi.device_error_flags() == 0


def test_static_scratch_rejects_problems_over_the_limit():
    # 262,144^2 at d 64 needs about 8 MB of partials: more than the 4 MiB array. Rejected before any launch.
    rows = m = 262_144
    assert _capi.workspace_size(rows, m, 64, _capi.PATH_TC) > _capi.lib.trnopt_static_scratch_bytes()
    t = torch.zeros(256, device="cuda")
    with pytest.raises(_capi.TrnoptError, match="static array"):
        _capi.half_step_tc_static(t, t, None, t, t, t, rows, m, 64, 0, 0, 0.1, 1.0, t)
