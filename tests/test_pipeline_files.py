"""Per-pair potential files and the resumable trajectory loop (trnopt.singlecell.save_pair / load_pair /
wot_trajectory), host side: the solve is replaced by a deterministic stand-in, so these run on the CPU. The real
solves through the same loop are in test_gpu_solver.py."""

import numpy as np
import pytest

import trnopt.singlecell as SC
from trnopt import SinkhornResult


def fake_map(x0, x1, growth=None, delta_days=1.0, **kw):
    """A TransportMap whose numbers depend on the inputs only (stands in for wot_transport_map)."""
    I, J = len(x0), len(x1)
    f, g = x0.sum(1) * 0.5, x1.sum(1) * -0.25
    G = np.ones(I) if growth is None else np.power(np.asarray(growth, dtype=np.float64), delta_days)
    res = SinkhornResult(f=f, g=g, iterations=7 * I, error=1e-9, converged=True, cost=1.0, seconds=0.01,
                         eps=kw.get("eps", 0.05), rho=(1.0, 50.0), center=x0.mean(0), cost_scale=2.5,
                         row_mass=G / I, col_mass=np.full(J, 1.0 / J))
    return SC.TransportMap(result=res, learned_growth=[G, 2 * G], seconds=0.01, iterations=7 * I)


def cohorts(sizes=(30, 41, 25, 33), d=4, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.normal(size=(n, d)) + k for k, n in enumerate(sizes)], [rng.random(n) + 0.5 for n in sizes]


def test_pair_file_round_trip_has_the_reference_keys(tmp_path):
    cs, gr = cohorts()
    tm = fake_map(cs[0], cs[1], gr[0], 0.5, eps=0.05)
    path = SC.save_pair(SC.pair_path(tmp_path, 3.5, 4.0), tm, cs[0], cs[1], cells1=[f"c{i}" for i in range(41)])
    assert path.name == "pair_3.5_4.npz" and not list(tmp_path.glob("*.partial"))
    with np.load(path) as z:                          # no pickled objects: loads with allow_pickle=False
        assert set(SC.PAIR_KEYS) <= set(z.files)
        assert z["cells1"][3] == "c3" and z["cells0"][2] == "2"
    sp = SC.load_pair(path)
    r, r2 = tm.result, sp.tm.result
    for k in ("f", "g", "center", "row_mass", "col_mass"):
        np.testing.assert_array_equal(getattr(r2, k), getattr(r, k))
    assert (r2.eps, r2.cost_scale, r2.rho, r2.iterations, r2.converged) == (0.05, 2.5, (1.0, 50.0), 7 * 30, True)
    np.testing.assert_array_equal(np.array(sp.tm.learned_growth), np.array(tm.learned_growth))
    np.testing.assert_array_equal(sp.x0, cs[0])
    assert sp.tm.iterations == tm.iterations


def test_reads_a_file_in_the_reference_examples_layout(tmp_path):
    """The reference example writes exactly PAIR_KEYS, cell names as object arrays (obs_names values)."""
    cs, _ = cohorts()
    rng = np.random.default_rng(1)
    path = tmp_path / "pair_16_16.5.npz"
    names0 = np.array([f"cell{i}" for i in range(30)], dtype=object)
    np.savez(path, f=rng.normal(size=30), g=rng.normal(size=41), eps=0.05, center=rng.normal(size=4),
             cost_scale=3.0, row_mass=rng.random(30), col_mass=rng.random(41),
             learned_growth=np.array([np.ones(30), rng.random(30)]), cells0=names0,
             cells1=np.array([f"d{i}" for i in range(41)], dtype=object), x0=cs[0], x1=cs[1])
    with pytest.raises(ValueError):
        SC.load_pair(path)                            # object arrays need an explicit allow_pickle
    sp = SC.load_pair(path, allow_pickle=True)
    assert sp.cells0[5] == "cell5" and sp.tm.result.rho is None and sp.tm.iterations == 0
    assert len(sp.tm.learned_growth) == 2 and sp.tm.result.f.shape == (30,)
    bad = tmp_path / "other.npz"
    np.savez(bad, f=np.zeros(3))
    with pytest.raises(ValueError, match="not a pair file"):
        SC.load_pair(bad)


def test_trajectory_saves_every_pair_and_resumes_at_the_first_missing_one(tmp_path, monkeypatch):
    calls = []
    monkeypatch.setattr(SC, "wot_transport_map", lambda *a, **k: calls.append(a[2] is not None) or fake_map(*a, **k))
    cs, gr = cohorts()
    times = [0.0, 0.5, 1.5, 2.0]
    first = SC.wot_trajectory(cs, times, gr, save=tmp_path, eps=0.05)
    assert len(calls) == 3
    assert sorted(p.name for p in tmp_path.iterdir()) == ["pair_0.5_1.5.npz", "pair_0_0.5.npz", "pair_1.5_2.npz"]
    # the growth of pair k is growth[k] ** (t1 - t0)
    np.testing.assert_allclose(first[1].result.row_mass * len(cs[1]), gr[1] ** 1.0)
    np.testing.assert_allclose(first[0].result.row_mass * len(cs[0]), gr[0] ** 0.5)
    # a run killed after the first pair: the other files are missing, the restart solves only those
    (tmp_path / "pair_0.5_1.5.npz").unlink()
    (tmp_path / "pair_1.5_2.npz").unlink()
    calls.clear()
    again = SC.wot_trajectory(cs, times, gr, save=tmp_path, resume=True, eps=0.05)
    assert len(calls) == 2
    for a, b in zip(first, again):
        np.testing.assert_array_equal(a.result.f, b.result.f)
        np.testing.assert_array_equal(a.result.g, b.result.g)
    # everything on file: nothing solved
    calls.clear()
    SC.wot_trajectory(cs, times, gr, save=tmp_path, resume=True, eps=0.05)
    assert calls == []
    # a file written for other coordinates is an error, not a silent reuse
    cs2 = [c.copy() for c in cs]
    cs2[2][0, 0] += 1.0
    with pytest.raises(ValueError, match="other coordinates"):
        SC.wot_trajectory(cs2, times, gr, save=tmp_path, resume=True, eps=0.05)


def test_trajectory_argument_checks(tmp_path):
    cs, gr = cohorts()
    with pytest.raises(ValueError, match="needs save"):
        SC.wot_trajectory(cs, resume=True)
    with pytest.raises(ValueError, match="times"):
        SC.wot_trajectory(cs, [0.0, 1.0])
    with pytest.raises(ValueError, match="growth"):
        SC.wot_trajectory(cs, None, gr[:2])
