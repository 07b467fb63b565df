"""Plan evaluation kernels (trnopt_plan_rows, trnopt_plan_log_row_sums) against the reference's float64 host
evaluation: the committed fixtures of its transport_plan, masses_from_potentials and ancestor pull-back, and the
oracle on seeded cases with ragged sizes. Float64 throughout, so the tolerances are near rounding level."""

import numpy as np
import pytest
import torch

from oracle import trnopt_oracle as O
from trnopt import _capi, plan, synthetic

pytestmark = pytest.mark.gpu

PLAN_RTOL = 1e-11      # plan entries and sums: float64 with a different summation order than NumPy
PULL_ATOL = 1e-10      # normalized log pull-back


def _wot_small(golden):
    z = golden("wot_small.npz")
    x0, x1, _ = synthetic.cfg3(n=735, m=896)
    r = O.Result(f=z["f"], g=z["g"], iterations=0, error=0.0, converged=True, cost=float("nan"), seconds=0.0,
                 eps=0.05, rho=(1.0, 50.0), center=z["center"], cost_scale=float(z["cost_scale"]))
    return x0, x1, r


def test_plan_rows_match_reference(golden):
    p = golden("plan_cases.npz")
    x0, x1, r = _wot_small(golden)
    a, b = np.full(len(x0), 1 / len(x0)), np.full(len(x1), 1 / len(x1))
    np.testing.assert_allclose(plan.plan_rows(x0, x1, r, p["rows"], a, b), p["plan_rows"], rtol=PLAN_RTOL, atol=0)
    P = plan.transport_plan(x0, x1, r, a, b)
    np.testing.assert_allclose(P.sum(1), p["plan_row_sum"], rtol=PLAN_RTOL)
    np.testing.assert_allclose(P.sum(0), p["plan_col_sum"], rtol=PLAN_RTOL)
    # negative indices count from the end, as NumPy does
    np.testing.assert_array_equal(plan.plan_rows(x0, x1, r, [-1, -735], a, b), P[[734, 0]])


def test_plan_marginals_match_reference(golden):
    p = golden("plan_cases.npz")
    x0, x1, r = _wot_small(golden)
    a, b = np.full(len(x0), 1 / len(x0)), np.full(len(x1), 1 / len(x1))
    rows, cols = plan.plan_marginals(x0, x1, r, a, b)
    np.testing.assert_allclose(rows, p["plan_row_sum"], rtol=PLAN_RTOL)
    np.testing.assert_allclose(cols, p["plan_col_sum"], rtol=PLAN_RTOL)
    s = np.sqrt(r.cost_scale)
    mr, mc = plan.masses_from_potentials((x0 - r.center) / s, (x1 - r.center) / s, a, b, r.f, r.g, 0.05)
    np.testing.assert_allclose(mr, p["masses_rows"], rtol=PLAN_RTOL)
    np.testing.assert_allclose(mc, p["masses_cols"], rtol=PLAN_RTOL)


@pytest.mark.parametrize("tag", ["smooth", "subset"])
def test_pull_back_matches_reference(golden, tag):
    """The subset case has log v = -inf outside 100 cells (columns that contribute nothing)."""
    p = golden("plan_cases.npz")
    x0, x1, r = _wot_small(golden)
    pb = plan.pull_back(x0, x1, r, p[f"log_v1_{tag}"])
    np.testing.assert_allclose(pb, p[f"pull_back_{tag}"], rtol=0, atol=PULL_ATOL)


@pytest.mark.parametrize("n,m,d", [(1, 1, 1), (63, 65, 3), (130, 77, 33), (257, 300, 70), (64, 128, 32)])
def test_plan_ragged_shapes_match_oracle(n, m, d):
    """Tile edges in rows and columns, coordinate chunks of 32 (d = 32, 33, 70), weights and offsets not uniform."""
    rng = np.random.default_rng(n * 1000 + m + d)
    x, y = rng.normal(size=(n, d)), rng.normal(size=(m, d)) * 0.7 + 0.2
    a, b = rng.random(n) + 0.1, rng.random(m) + 0.1
    r = O.Result(f=rng.normal(size=n), g=rng.normal(size=m), iterations=0, error=0.0, converged=True,
                 cost=float("nan"), seconds=0.0, eps=0.7, rho=None, center=rng.normal(size=d) * 0.1,
                 cost_scale=1.3)
    P = O.transport_plan(x, y, r, a, b)
    np.testing.assert_allclose(plan.transport_plan(x, y, r, a, b), P, rtol=PLAN_RTOL, atol=1e-300)
    rows, cols = plan.plan_marginals(x, y, r, a, b)
    np.testing.assert_allclose(rows, P.sum(1), rtol=PLAN_RTOL)
    np.testing.assert_allclose(cols, P.sum(0), rtol=PLAN_RTOL)


def test_log_row_sums_survive_underflow():
    """Rows whose every entry underflows exp() in float64 still get their log sum (the reference's pull-back takes
    logsumexp for the same reason)."""
    rng = np.random.default_rng(3)
    x, y = rng.normal(size=(200, 8)), rng.normal(size=(150, 8))
    f, g = rng.normal(size=200) - 60.0, rng.normal(size=150) - 60.0
    eps = 0.05
    dev = torch.device("cuda", torch.cuda.current_device())
    t = lambda v: torch.as_tensor(np.ascontiguousarray(v, dtype=np.float64), device=dev)
    got = _capi.plan_log_row_sums(t(x), t(y), t(f), t(g), None, None, eps).cpu().numpy()
    from scipy.special import logsumexp
    C = ((x[:, None, :] - y[None, :, :]) ** 2).sum(2)
    want = f / eps + logsumexp((g[None, :] - C) / eps, axis=1)
    assert np.all(want < -745)              # exp() of every entry is 0 in float64
    np.testing.assert_allclose(got, want, rtol=1e-13)


def test_plan_log_row_sums_deterministic():
    x0, x1, _ = synthetic.cfg3(n=1500, m=1700)
    dev = torch.device("cuda", torch.cuda.current_device())
    t = lambda v: torch.as_tensor(np.ascontiguousarray(v, dtype=np.float64), device=dev)
    rng = np.random.default_rng(1)
    args = (t(x0 / 8), t(x1 / 8), t(rng.normal(size=1500)), t(rng.normal(size=1700)), None, None, 0.2)
    a, b = _capi.plan_log_row_sums(*args), _capi.plan_log_row_sums(*args)
    assert torch.equal(a, b)


def test_plan_row_index_checks():
    x, y = np.zeros((10, 3)), np.ones((7, 3))
    r = O.Result(f=np.zeros(10), g=np.zeros(7), iterations=0, error=0.0, converged=True, cost=0.0, seconds=0.0,
                 eps=1.0, rho=None, center=np.zeros(3), cost_scale=1.0)
    with pytest.raises(IndexError):
        plan.plan_rows(x, y, r, [10])
    with pytest.raises(IndexError):
        plan.plan_rows(x, y, r, [-11])
    # the C ABI itself turns an out-of-range device index into a NaN row and reads nothing for it
    dev = torch.device("cuda", torch.cuda.current_device())
    t = lambda v: torch.as_tensor(v, dtype=torch.float64, device=dev)
    out = _capi.plan_rows(t(x), t(y), None, None, None, None, 1.0,
                          torch.tensor([2, 10, -1, 3], dtype=torch.int32, device=dev)).cpu().numpy()
    assert np.all(np.isnan(out[1])) and np.all(np.isnan(out[2]))
    np.testing.assert_allclose(out[0], np.exp(-3.0), rtol=1e-15)
    np.testing.assert_allclose(out[3], np.exp(-3.0), rtol=1e-15)
    with pytest.raises(_capi.TrnoptError):
        _capi.plan_rows(t(x), t(y), None, None, None, None, 0.0, torch.tensor([0], dtype=torch.int32, device=dev))


def test_plan_marginals_at_cfg2_size():
    """Size-independent properties at 10,000^2, d 64 (config 2's clouds): the row sums and the column sums of one
    plan carry the same total mass, and the row sums of a converged balanced solve are its marginal a = 1/n."""
    from trnopt import Backend, SinkhornOptions, sinkhorn
    x, y = synthetic.cfg2()
    r = sinkhorn(x, y, opts=SinkhornOptions(eps=0.1, max_iters=2000, tol=1e-6, normalize=False,
                                            backend=Backend.preset("cuda-fused")))
    rows, cols = plan.plan_marginals(x, y, r)
    assert abs(rows.sum() / cols.sum() - 1) < 1e-12
    # after the g update the column sums are b up to float64 evaluation of fp32 potentials
    assert np.abs(cols * len(y) - 1).max() < 2e-3
    assert np.abs(rows * len(x) - 1).sum() / len(x) < 1e-5 * 50


@pytest.mark.parametrize("tag", list(synthetic.PCA_CASES))
def test_local_pca_coords_match_reference(golden, tag):
    """GPU local PCA (wot's per-pair embedding) against the reference's local_pca_coords on the same seeded
    expression, for each solver sklearn's PCA picks (randomized, transposed randomized, full, covariance-eigh)."""
    from trnopt.singlecell import local_pca_coords
    z = golden("pca_cases.npz")
    c0, c1, genes, seed = synthetic.PCA_CASES[tag]
    e0, e1 = synthetic.expression(c0, c1, genes, seed)
    p0, p1 = local_pca_coords(e0, e1, 30)
    scale = np.abs(z[f"{tag}_p0"]).max()
    np.testing.assert_allclose(p0, z[f"{tag}_p0"], rtol=0, atol=1e-8 * scale)
    np.testing.assert_allclose(p1, z[f"{tag}_p1"], rtol=0, atol=1e-8 * scale)
