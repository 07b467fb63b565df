"""bench.py's roofline arithmetic on CPU: the exp bound counts the unpadded n * m (per GPU: n / N rows against all m
columns), the fraction is achieved exps/s over 148 SMs x 16 ex2/clk x the max SM clock, the slowest of the three
bounds is named, and the DRAM traffic comes from the committed ncu capture of the same kernel and workload (none for
an N-GPU shard without its own capture)."""

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_exp_bound_counts_unpadded_pairs(bench):
    n = m = 10_000
    pk, _ = bench.peaks()
    mhz = pk.get("sm_max_mhz", 1965.0)
    launch_ms = 0.047
    r = bench.roofline(n, m, 64, 1, launch_ms, "tc", None, None, None)
    exp_peak = 148 * 16 * mhz * 1e6
    assert r["bound"] == "exp" and r["unit"] == "exp/s"
    assert r["per_launch"]["exps"] == n * m
    assert r["achieved"] == pytest.approx(n * m / (launch_ms * 1e-3))
    assert r["frac"] == pytest.approx(n * m / (launch_ms * 1e-3) / exp_peak, abs=1e-4)
    assert r["bounds_us"]["exp"] == pytest.approx(n * m / exp_peak * 1e6, rel=1e-3)
    assert r["slowest"] == "exp"                       # config 2 is exp-bound, not contraction- or HBM-bound
    assert r["per_launch"]["useful_flops"] == 2.0 * n * m * 64


def test_shards_divide_the_rows_and_add_the_nvlink_bound(bench):
    n = m = 262_144
    one = bench.roofline(n, m, 64, 1, 27.0, "tc", None, None, None)
    eight = bench.roofline(n, m, 64, 8, 3.2, "tc", None, None, None)
    assert eight["per_launch"]["exps"] == n * m / 8
    assert "nvlink" in eight["bounds_us"] and "nvlink" not in one["bounds_us"]
    assert eight["per_launch"]["nvlink_bytes_out"] == pytest.approx(n / 8 * 4 * 7)


def test_traffic_comes_from_the_matching_capture(bench):
    t2, src2 = bench.measured_traffic("tc", "cfg2", 1)
    t5, _ = bench.measured_traffic("tc", "cfg5", 1)
    assert t2 is not None and 5e6 < t2 < 6e6 and "traffic_tc_cfg2.json" in src2   # ~ the 5.4 MB algorithmic bytes
    assert t5 is not None and t5 < 2e9                                             # the common sweep phase's capture
    assert bench.measured_traffic("tc", "cfg5", 8) == (None, None)
