"""The fused half-step through the C ABI against the reference's own answers (golden KATs) and the float64 oracle.

Tolerance: potentials are compared in units of eps, |fh_gpu - fh_ref| / eps <= HS_TOL, or, on the reference's own
known-answer inputs, no worse than the reference's float32 half-step on the same inputs (its uncentred case with
eps 0.02 has scores of magnitude ~300, where one float32 rounding is already ~2e-5 eps). Both kernels (FFMA and
tensor-core split precision) are held to the same bar.
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


PATHS = [_capi.PATH_FFMA, _capi.PATH_TC]
PATH_IDS = ["ffma", "tc"]


def scale_exp(a):
    mx = float(np.abs(a).max())
    return 0 if mx == 0 else 14 - int(np.ceil(np.log2(mx)))


def gpu_half_step(x, xsq, off, y, gh, log_b, eps, kappa, ws=None, path=_capi.PATH_FFMA):
    rows, d = x.shape
    m = y.shape[0]
    xT, ldx = _capi._pad_ld(_dev(x.T))
    yT, ldy = _capi._pad_ld(_dev(y.T))
    if ws is None:
        ws = _capi.new_workspace(_capi.workspace_size(rows, m, d, path), "cuda")
    fh = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    offd = None if off is None else _dev(off)
    if path == _capi.PATH_FFMA:
        _capi.half_step(xT, ldx, _dev(xsq), offd, yT, ldy, _dev(gh), _dev(log_b), rows, m, d, eps, kappa, fh, ws)
    else:
        sx, sy = scale_exp(x), scale_exp(y)
        xp = _capi.pack_cloud(xT, ldx, rows, d, sx)
        yp = _capi.pack_cloud(yT, ldy, m, d, sy)
        _capi.half_step_tc(xp, _dev(xsq), offd, yp, _dev(gh), _dev(log_b), rows, m, d, sx, sy, eps, kappa, fh, ws)
    torch.cuda.synchronize()
    assert _capi.device_error_flags() == 0
    return fh.cpu().numpy().astype(np.float64)


def oracle_half_step(x, xsq, off, y, gh, log_b, eps, kappa):
    t = lambda a: torch.as_tensor(a, dtype=torch.float64)
    off = np.zeros(len(x)) if off is None else off
    return O.half_step(t(x), t(xsq), t(off), t(y.T.copy()), t(gh), t(log_b), 1.0 / eps, eps, kappa).numpy()


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_half_step_reference_kat(golden, path):
    z = golden("half_step_kat.npz")
    for c in range(int(z["ncases"])):
        g = lambda k: z[f"c{c}_{k}"]
        eps, kappa = float(g("eps")), float(g("kappa"))
        if path == _capi.PATH_TC and not _capi.tc_supported(g("x").shape[1]):
            continue
        fh = gpu_half_step(g("x"), g("xsq"), g("off"), g("y"), g("gh"), g("log_b"), eps, kappa, path=path)
        err = np.abs(fh - g("fh_f64")).max() / eps
        ref32 = np.abs(g("fh_f32") - g("fh_f64")).max() / eps
        assert err <= max(HS_TOL, ref32), (c, err, ref32)


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
    (1000, 2000, 30, 0.05, 1.0, True, 0),        # d <= 32 kernel, a row tile over 8 CTAs: 16 partials in one round
    (1000, 257, 128, 0.1, 1.0, False, 1),
    (4096, 4096, 64, 0.02, 0.7, True, 96),
    (20000, 700, 64, 0.1, 1.0, False, 0),
])
@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_half_step_matches_oracle(rows, m, d, eps, kappa, use_off, pad, path):
    if path == _capi.PATH_TC and not _capi.tc_supported(d):
        pytest.skip("tensor-core path covers d <= 64")
    x, xsq, off, y, gh, lb = problem(rows, m, d, rows * 7 + m, eps, pad)
    off = off if use_off else None
    fh = gpu_half_step(x, xsq, off, y, gh, lb, eps, kappa, path=path)
    ref = oracle_half_step(x, xsq, off, y, gh, lb, eps, kappa)
    err = np.abs(fh - ref).max() / eps
    assert np.all(np.isfinite(fh)) and err <= HS_TOL, err


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_padding_columns_before_real_ones(path):
    """Zero-weight (log_b = -1e9) columns ahead of the real ones: the running max first settles on a padding score
    near -1.4e9 and must recover full precision when the real columns arrive (any caller may order columns so)."""
    rows, m, d, eps = 700, 3000, 30, 0.05
    x, xsq, off, y, gh, lb = problem(rows, m, d, 5, eps)
    lb[:700] = -1e9
    fh = gpu_half_step(x, xsq, off, y, gh, lb, eps, 0.95, path=path)
    ref = oracle_half_step(x, xsq, off, y, gh, lb, eps, 0.95)
    err = np.abs(fh - ref).max() / eps
    assert np.all(np.isfinite(fh)) and err <= HS_TOL, err


def test_tc_and_ffma_agree_at_config_2_size():
    """One full-size config-2 half-step (10k x 10k, d 64, centred U[0,1] points) on both kernels."""
    from trnopt import synthetic
    x, y = synthetic.cfg2()
    c = np.concatenate([x, y]).mean(0)
    x, y = x - c, y - c
    gh = -(y * y).sum(1)
    lb = np.full(len(y), -np.log(len(y)))
    a = gpu_half_step(x, (x * x).sum(1), None, y, gh, lb, 0.1, 1.0, path=_capi.PATH_FFMA)
    b = gpu_half_step(x, (x * x).sum(1), None, y, gh, lb, 0.1, 1.0, path=_capi.PATH_TC)
    rows = np.random.default_rng(0).choice(len(x), 64, replace=False)
    ref = oracle_half_step(x[rows], (x[rows] ** 2).sum(1), None, y, gh, lb, 0.1, 1.0)
    assert np.abs(a[rows] - ref).max() / 0.1 <= HS_TOL
    assert np.abs(b[rows] - ref).max() / 0.1 <= HS_TOL
    assert np.abs(a - b).max() / 0.1 <= 2 * HS_TOL


@pytest.mark.parametrize("rows", [128, 2000])
def test_large_column_cloud_in_common_sweep_order(rows):
    """A column cloud over 32 MB packed (140,001 columns at d 64, a ragged last column tile) is swept by every CTA in
    a common phase, each row tile starting at its own rotation: one row tile spread over all CTAs (the rotation taken
    from a CTA more than 31 ranges away) and 16 row tiles of ~9 CTAs each, against the oracle on 64 sampled rows."""
    m, d, eps = 140_001, 64, 0.05
    assert m * 2 * d * 2 > 32 << 20
    x, xsq, off, y, gh, lb = problem(rows, m, d, 11 + rows, eps)
    fh = gpu_half_step(x, xsq, off, y, gh, lb, eps, 1.0, path=_capi.PATH_TC)
    pick = np.random.default_rng(rows).choice(rows, 64, replace=False)
    ref = oracle_half_step(x[pick], xsq[pick], off[pick], y, gh, lb, eps, 1.0)
    err = np.abs(fh[pick] - ref).max() / eps
    assert np.all(np.isfinite(fh)) and err <= HS_TOL, err


def test_fma_pipe_exp2_against_cuda_exp2f():
    """The FMA-pipe 2^x (range reduction + degree-5 polynomial fitted for this library) against CUDA's exp2f
    (torch.exp2 on the GPU) and against float64: relative error within 3e-7 over [-125, 100]. Evaluated through the
    packed pair form the fold uses; the test kernel returns NaN wherever the two lanes or the scalar form differ."""
    x = torch.cat([torch.linspace(-125, 100, 1_000_001), torch.linspace(-1, 1, 100_001)]).cuda()
    got = _capi.test_ex2_poly(x)
    ref_cuda = torch.exp2(x)
    ref64 = torch.exp2(x.double())
    assert ((got.double() / ref64 - 1).abs().max().item()) <= 3e-7
    assert ((got / ref_cuda - 1).abs().max().item()) <= 5e-7
    assert _capi.test_ex2_poly(torch.tensor([-1e9, -float("inf")], device="cuda")).max().item() < 1e-37


def test_row_lse_reference_kat(golden):
    z = golden("row_lse_kat.npz")
    lse = _capi.row_lse(_dev(z["xa_T"]), _dev(z["ya_T"])).cpu().numpy()
    assert np.abs(lse - z["lse"]).max() <= LSE_TOL


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_workspace_is_left_ready_and_results_are_deterministic(path):
    x, xsq, off, y, gh, lb = problem(3000, 7000, 64, 1, 0.1)
    ws = _capi.new_workspace(_capi.workspace_size(3000, 7000, 64, path), "cuda")
    a = gpu_half_step(x, xsq, off, y, gh, lb, 0.1, 0.9, ws=ws, path=path)
    b = gpu_half_step(x, xsq, off, y, gh, lb, 0.1, 0.9, ws=ws, path=path)
    assert np.array_equal(a, b)
    assert torch.count_nonzero(ws[:256]).item() == 0          # arrival counters back at zero
    assert _capi.device_error_flags() == 0


def _half_step_f64_on_gpu(x, xsq, off, y, gh, log_b, eps, kappa):
    """The half-step (sinkhorn.py:108-119) in float64 with torch on the GPU, for sizes the CPU oracle is slow at."""
    t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.float64), device="cuda")
    X, Y = t(x), t(y)
    z = (2.0 * X @ Y.T + t(gh)[None, :]) / eps + t(log_b)[None, :]
    lse = torch.logsumexp(z, dim=1)
    off = np.zeros(len(x)) if off is None else off
    return (kappa * (t(xsq) + eps * t(off) - eps * lse) - t(xsq)).cpu().numpy()


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_calls_of_different_shapes_share_a_workspace(path):
    """The f and g half-steps of a solve share one workspace although their row-tile counts differ (here 64 and
    70 tiles, on either side of a 64-counter block): every row of every output is checked, twice round."""
    n, m, d, eps = 8142, 8930, 16, 0.1
    x, xsq, off, y, gh, lb = problem(n, m, d, 3, eps)
    ysq = (y * y).sum(1)
    la = np.full(n, -np.log(n))
    ws = _capi.new_workspace(max(_capi.workspace_size(n, m, d, path), _capi.workspace_size(m, n, d, path)), "cuda")
    for _ in range(2):
        fh = gpu_half_step(x, xsq, off, y, gh, lb, eps, 0.9, ws=ws, path=path)
        ref = _half_step_f64_on_gpu(x, xsq, off, y, gh, lb, eps, 0.9)
        assert np.abs(fh - ref).max() / eps <= HS_TOL
        gh = gpu_half_step(y, ysq, None, x, fh, la, eps, 1.0, ws=ws, path=path)
        ref = _half_step_f64_on_gpu(y, ysq, None, x, fh, la, eps, 1.0)
        assert np.abs(gh - ref).max() / eps <= HS_TOL


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
