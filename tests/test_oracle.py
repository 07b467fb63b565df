"""The CPU oracle (oracle/trnopt_oracle.py) pinned against the reference's own outputs (tests/golden/, written by
tests/golden/make_golden.py from the reference run in the build container). CPU only."""

import numpy as np
import pytest
import torch

from oracle import trnopt_oracle as O
from trnopt import synthetic


def clouds(n=137, m=91, d=5, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(size=(n, d)), rng.normal(size=(m, d)) * 0.8 + 0.5


def test_half_step_matches_reference_kat(golden):
    z = golden("half_step_kat.npz")
    for c in range(int(z["ncases"])):
        g = lambda k: z[f"c{c}_{k}"]
        eps, kappa = float(g("eps")), float(g("kappa"))
        for tag, dt, tol in (("f64", torch.float64, 1e-12), ("f32", torch.float32, 1e-6)):
            t = lambda a: torch.as_tensor(a, dtype=dt)
            fh = O.half_step(t(g("x")), t(g("xsq")), t(g("off")), t(g("y").T.copy()), t(g("gh")), t(g("log_b")),
                             t(1.0 / eps), t(eps), t(kappa)).numpy()
            ref = g(f"fh_{tag}")
            assert np.abs(fh - ref).max() / eps <= tol * max(1.0, np.abs(ref).max()), (c, tag)


def test_row_lse_kat(golden):
    z = golden("row_lse_kat.npz")
    lse = O.row_lse_np(z["xa_T"], z["ya_T"])
    np.testing.assert_allclose(lse, z["lse"], rtol=0, atol=1e-12)


def _cmp(res, z, prefix, atol_pot=1e-9):
    meta = z[prefix + "_meta"]
    assert res.iterations == int(meta[0]), prefix
    assert bool(res.converged) == bool(meta[2]), prefix
    np.testing.assert_allclose(res.f, z[prefix + "_f"], rtol=0, atol=atol_pot)
    np.testing.assert_allclose(res.g, z[prefix + "_g"], rtol=0, atol=atol_pot)
    if prefix + "_row_mass" in z:
        np.testing.assert_allclose(res.row_mass, z[prefix + "_row_mass"], rtol=1e-9)
        np.testing.assert_allclose(res.col_mass, z[prefix + "_col_mass"], rtol=1e-9)


def test_solver_matches_reference_cases(golden):
    z = golden("solver_cases.npz")
    x, y = clouds()
    o = dict(eps=0.1, tol=1e-7, max_iters=5000)
    _cmp(O.solve(x, y, opts=O.Options(**o)), z, "balanced_f64")
    _cmp(O.solve(x, y, opts=O.Options(block=32, block_y=40, **o)), z, "blocked_f64")
    a = np.random.default_rng(1).uniform(0.5, 1.5, len(x)) / len(x)
    _cmp(O.solve(x, y, a=a, opts=O.Options(rho=1.0, block=50, **o)), z, "unbalanced_f64")
    rng = np.random.default_rng(2)
    wa = rng.uniform(0.2, 1.0, len(x)); wa /= wa.sum()
    wb = rng.uniform(0.2, 1.0, len(y)); wb /= wb.sum()
    _cmp(O.solve(x, y, wa, wb, O.Options(**o)), z, "weighted_f64")
    _cmp(O.solve(x, y, opts=O.Options(max_iters=7, fixed_iters=True)), z, "fixed7_f64")
    x2, y2 = clouds(n=90, m=70, d=4, seed=7)
    G = np.random.default_rng(8).uniform(0.5, 2.0, len(x2))
    I, J = len(x2), len(y2)
    for staged in (False, True):
        so = O.Options(eps=0.2, rho=(1.0, 50.0), normalize="median", tol=1e-8, max_iters=20_000, check_every=5,
                       eps_stages=O.wot_eps_stages(0.2) if staged else None)
        r = O.solve(x2, y2, np.full(I, 1 / I), np.full(J, 1 / J), so, a_target=G / I, b_target=np.full(J, G.mean() / J))
        _cmp(r, z, f"wot{'_staged' if staged else ''}_f64")


def test_solver_float32_matches_reference_float32(golden):
    """Same CPU float32 workload as the reference's cpu-float32 preset (the timed CPU baseline)."""
    z = golden("solver_cases.npz")
    x, y = clouds()
    r = O.solve(x, y, opts=O.Options(eps=0.1, tol=1e-5, max_iters=5000, dtype=torch.float32))
    _cmp(r, z, "balanced_f32", atol_pot=1e-6)


def test_eps_scaling_cases(golden):
    z = golden("solver_cases.npz")
    x3, y3 = clouds(n=300, m=250, d=10, seed=3)
    o = dict(eps=0.01, tol=1e-6, max_iters=20_000)
    _cmp(O.solve(x3, y3, opts=O.Options(eps_start=2.0, eps_decay=0.8, **o)), z, "epsscaled_f64")


def test_rejects_unequal_mass_when_balanced():
    x, y = clouds()
    with pytest.raises(ValueError):
        O.solve(x, y, a=np.full(len(x), 2.0 / len(x)))


def test_normalization_matches_reference(golden):
    z = golden("normalization.npz")
    for tag, n, m, d, seed in [("a", 137, 91, 5, 0), ("b", 90, 70, 4, 7), ("c", 301, 250, 10, 3),
                               ("d", 1000, 1200, 30, 11)]:
        x, y = clouds(n, m, d, seed)
        for how in ("mean", "median"):
            c, s = O.normalization(x, y, how=how)
            np.testing.assert_array_equal(c, z[f"{tag}_{how}_center"])
            assert s == float(z[f"{tag}_{how}_scale"])


def test_cfg3_median_matches_reference(golden):
    z = golden("normalization.npz")
    x0, x1, _ = synthetic.cfg3()
    c, s = O.normalization(x0, x1, how="median")
    np.testing.assert_array_equal(c, z["cfg3_median_center"])
    assert s == float(z["cfg3_median_scale"])


def test_cfg1_oracle_matches_reference(golden):
    """Config 1 (2,000^2, d 16, 200 fixed iterations) through the oracle in float64: the reference's answer."""
    z = golden("cfg1.npz")
    x, y = synthetic.cfg1()
    r = O.solve(x, y, opts=O.Options(eps=0.1, max_iters=200, fixed_iters=True, normalize=False))
    np.testing.assert_allclose(r.f, z["f_f64"], rtol=0, atol=1e-10)
    np.testing.assert_allclose(r.g, z["g_f64"], rtol=0, atol=1e-10)
    rows, cols = O.plan_marginals(x, y, r.f, r.g, 0.1, r.center, r.cost_scale)
    np.testing.assert_allclose(rows, z["row_sum_f64"], rtol=1e-10)
    np.testing.assert_allclose(cols, z["col_sum_f64"], rtol=1e-10)


def test_wot_small_matches_reference(golden):
    z = golden("wot_small.npz")
    x0, x1, growth = synthetic.cfg3(n=735, m=896)
    res, learned, iters = O.wot_transport_map(x0, x1, growth, eps=0.05, lambda1=1.0, lambda2=50.0, growth_iters=3,
                                              tol=1e-8)
    assert iters == int(z["iterations"])
    np.testing.assert_allclose(res.row_mass, z["row_mass"], rtol=1e-9)
    np.testing.assert_allclose(res.col_mass, z["col_mass"], rtol=1e-9)
    np.testing.assert_allclose(res.f, z["f"], rtol=0, atol=1e-9)


def _wot_small_result(z):
    return O.Result(f=z["f"], g=z["g"], iterations=0, error=0.0, converged=True, cost=float("nan"), seconds=0.0,
                    eps=0.05, rho=(1.0, 50.0), center=z["center"], cost_scale=float(z["cost_scale"]))


def test_plan_functions_match_reference(golden):
    """Oracle plan rows, plan sums, masses_from_potentials and the ancestor pull-back against the reference's own
    transport_plan and example functions on wot_small's potentials."""
    z, p = golden("wot_small.npz"), golden("plan_cases.npz")
    x0, x1, _ = synthetic.cfg3(n=735, m=896)
    I, J = len(x0), len(x1)
    r = _wot_small_result(z)
    a, b = np.full(I, 1.0 / I), np.full(J, 1.0 / J)
    P = O.transport_plan(x0, x1, r, a, b)
    np.testing.assert_allclose(P[p["rows"]], p["plan_rows"], rtol=1e-12, atol=0)
    rows, cols = O.plan_marginals(x0, x1, r.f, r.g, 0.05, r.center, r.cost_scale, a, b)
    np.testing.assert_allclose(rows, p["plan_row_sum"], rtol=1e-10)
    np.testing.assert_allclose(cols, p["plan_col_sum"], rtol=1e-10)
    s = np.sqrt(r.cost_scale)
    mr, mc = O.masses_from_potentials((x0 - r.center) / s, (x1 - r.center) / s, a, b, r.f, r.g, 0.05)
    np.testing.assert_allclose(mr, p["masses_rows"], rtol=1e-12)
    np.testing.assert_allclose(mc, p["masses_cols"], rtol=1e-12)
    for tag in ("smooth", "subset"):
        pb = O.pull_back(x0, x1, r.f, r.g, 0.05, r.center, r.cost_scale, p[f"log_v1_{tag}"])
        np.testing.assert_allclose(pb, p[f"pull_back_{tag}"], rtol=0, atol=1e-10)


def test_local_pca_matches_reference(golden):
    """The PCA restatement (randomized, transposed randomized, full and covariance-eigh solvers) against the
    reference's local_pca_coords run on the same seeded expression."""
    z = golden("pca_cases.npz")
    for tag, (c0, c1, genes, seed) in synthetic.PCA_CASES.items():
        e0, e1 = synthetic.expression(c0, c1, genes, seed)
        p0, p1 = O.local_pca_coords(e0, e1, 30)
        scale = np.abs(z[f"{tag}_p0"]).max()
        np.testing.assert_allclose(p0, z[f"{tag}_p0"], rtol=0, atol=1e-8 * scale, err_msg=tag)
        np.testing.assert_allclose(p1, z[f"{tag}_p1"], rtol=0, atol=1e-8 * scale, err_msg=tag)
