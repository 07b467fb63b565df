"""The fused half-step through the C ABI against the reference's own answers (golden KATs) and the float64 oracle.

Tolerance: potentials are compared in units of eps, |fh_gpu - fh_ref| / eps <= HS_TOL. The reference's own float32
half-step is about 1e-5 eps from its float64 one on these inputs; HS_TOL leaves room for a different (also
float32) summation order.
"""

import numpy as np
import pytest
import torch

from oracle import trnopt_oracle as O
from trnopt import _capi

pytestmark = pytest.mark.gpu
HS_TOL = 5e-5          # |delta fh| / eps
LSE_TOL = 2e-5         # |delta lse| (natural log units)


def _dev(a, dt=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).cuda()


def gpu_half_step(x, xsq, off, y, gh, log_b, eps, kappa, ws=None, path=_capi.PATH_FFMA):
    rows, d = x.shape
    m = y.shape[0]
    xT, ldx = _capi._pad_ld(_dev(x.T))
    yT, ldy = _capi._pad_ld(_dev(y.T))
    if ws is None:
        ws = _capi.new_workspace(_capi.workspace_size(rows, m, d, path), "cuda")
    fh = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    _capi.half_step(xT, ldx, _dev(xsq), None if off is None else _dev(off), yT, ldy, _dev(gh), _dev(log_b), rows, m,
                    d, eps, kappa, fh, ws)
    return fh.cpu().numpy().astype(np.float64)


def oracle_half_step(x, xsq, off, y, gh, log_b, eps, kappa):
    t = lambda a: torch.as_tensor(a, dtype=torch.float64)
    off = np.zeros(len(x)) if off is None else off
    return O.half_step(t(x), t(xsq), t(off), t(y.T.copy()), t(gh), t(log_b), 1.0 / eps, eps, kappa).numpy()


def test_half_step_reference_kat(golden):
    z = golden("half_step_kat.npz")
    for c in range(int(z["ncases"])):
        g = lambda k: z[f"c{c}_{k}"]
        eps, kappa = float(g("eps")), float(g("kappa"))
        fh = gpu_half_step(g("x"), g("xsq"), g("off"), g("y"), g("gh"), g("log_b"), eps, kappa)
        err = np.abs(fh - g("fh_f64")).max() / eps
        ref32 = np.abs(g("fh_f32") - g("fh_f64")).max() / eps
        assert err <= HS_TOL, (c, err, ref32)


def problem(rows, m, d, seed, eps, pad=0):
    """Inputs shaped like a solver's: centred points with costs O(1), a plausible shifted potential, padding."""
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(rows, d)) / np.sqrt(2 * d)
    y = rng.normal(size=(m, d)) / np.sqrt(2 * d) + 0.1 / np.sqrt(d)
    gh = -(y * y).sum(1) + rng.normal(scale=0.2, size=m)
    log_b = np.full(m, -np.log(max(1, m - pad)))
    if pad:
        y[m - pad:] = 0.0
        log_b[m - pad:] = -1e9
    return x, (x * x).sum(1), rng.normal(scale=0.3, size=rows), y, gh, log_b


@pytest.mark.parametrize("rows,m,d,eps,kappa,use_off,pad", [
    (1, 1, 1, 0.1, 1.0, False, 0),
    (1, 1000, 3, 0.05, 1.0, True, 0),
    (127, 129, 16, 0.1, 0.9, True, 5),
    (128, 128, 64, 0.1, 1.0, False, 0),
    (300, 5000, 30, 0.05, 0.98, True, 200),
    (1000, 257, 128, 0.1, 1.0, False, 1),
    (4096, 4096, 64, 0.02, 0.7, True, 96),
    (20000, 700, 64, 0.1, 1.0, False, 0),
])
def test_half_step_matches_oracle(rows, m, d, eps, kappa, use_off, pad):
    x, xsq, off, y, gh, lb = problem(rows, m, d, rows * 7 + m, eps, pad)
    off = off if use_off else None
    fh = gpu_half_step(x, xsq, off, y, gh, lb, eps, kappa)
    ref = oracle_half_step(x, xsq, off, y, gh, lb, eps, kappa)
    err = np.abs(fh - ref).max() / eps
    assert np.all(np.isfinite(fh)) and err <= HS_TOL, err


def test_row_lse_reference_kat(golden):
    z = golden("row_lse_kat.npz")
    lse = _capi.row_lse(_dev(z["xa_T"]), _dev(z["ya_T"])).cpu().numpy()
    assert np.abs(lse - z["lse"]).max() <= LSE_TOL


def test_workspace_is_left_ready_and_results_are_deterministic():
    x, xsq, off, y, gh, lb = problem(3000, 7000, 64, 1, 0.1)
    ws = _capi.new_workspace(_capi.workspace_size(3000, 7000, 64), "cuda")
    a = gpu_half_step(x, xsq, off, y, gh, lb, 0.1, 0.9, ws=ws)
    b = gpu_half_step(x, xsq, off, y, gh, lb, 0.1, 0.9, ws=ws)
    assert np.array_equal(a, b)
    assert torch.count_nonzero(ws[:256]).item() == 0          # arrival counters back at zero
    assert _capi.device_error_flags() == 0


def test_argument_errors_are_reported_not_launched():
    x, xsq, off, y, gh, lb = problem(10, 20, 4, 2, 0.1)
    xT, ldx = _capi._pad_ld(_dev(x.T))
    yT, ldy = _capi._pad_ld(_dev(y.T))
    fh = torch.empty(10, device="cuda")
    small = torch.zeros(8, dtype=torch.uint8, device="cuda")
    with pytest.raises(_capi.TrnoptError, match="workspace"):
        _capi.half_step(xT, ldx, _dev(xsq), None, yT, ldy, _dev(gh), _dev(lb), 10, 20, 4, 0.1, 1.0, fh, small)
    ws = _capi.new_workspace(_capi.workspace_size(10, 20, 4), "cuda")
    with pytest.raises(_capi.TrnoptError, match="invalid"):
        _capi.half_step(xT, ldx, _dev(xsq), None, yT, ldy, _dev(gh), _dev(lb), 10, 20, 4, -0.1, 1.0, fh, ws)
    with pytest.raises(_capi.TrnoptError, match="misaligned"):
        _capi.half_step(xT, ldx - 1, _dev(xsq), None, yT, ldy, _dev(gh), _dev(lb), 10, 20, 4, 0.1, 1.0, fh, ws)
    with pytest.raises(_capi.TrnoptError, match="unsupported"):
        _capi.half_step(xT, ldx, _dev(xsq), None, yT, ldy, _dev(gh), _dev(lb), 10, 20, 129, 0.1, 1.0, fh, ws)


def test_median_cost_matches_reference(golden):
    from trnopt import synthetic
    from trnopt.sinkhorn import normalization
    z = golden("normalization.npz")
    rng_cases = [("a", 137, 91, 5, 0), ("b", 90, 70, 4, 7), ("c", 301, 250, 10, 3), ("d", 1000, 1200, 30, 11)]
    for tag, n, m, d, seed in rng_cases:
        r = np.random.default_rng(seed)
        x, y = r.normal(size=(n, d)), r.normal(size=(m, d)) * 0.8 + 0.5
        c, s = normalization(x, y, how="median")
        np.testing.assert_array_equal(c, z[f"{tag}_median_center"])
        assert abs(s - float(z[f"{tag}_median_scale"])) <= 1e-14 * s, tag
    x0, x1, _ = synthetic.cfg3()
    c, s = normalization(x0, x1, how="median")
    assert abs(s - float(z["cfg3_median_scale"])) <= 1e-14 * s
