"""Host-side logic that needs no GPU: kernel selection and its errors, the padded cloud layout, the stream-K work
split used by the kernels, presets, eps stages and the synthetic generators. CPU only."""

import numpy as np
import pytest
import torch

from oracle import trnopt_oracle as O
from trnopt import Backend, SinkhornOptions, sinkhorn, synthetic
from trnopt import sinkhorn as sk_mod_fn  # noqa: F401  (the function; the module is below)
import trnopt.sinkhorn  # noqa: F401
import sys

S = sys.modules["trnopt.sinkhorn"]


def clouds(n=137, m=91, d=5, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(size=(n, d)), rng.normal(size=(m, d)) * 0.8 + 0.5


def test_presets_match_the_reference_table_plus_cuda_fused():
    assert Backend.preset("cuda-fused") == Backend(device="cuda", dtype=torch.float32)
    assert Backend.preset("cpu") == Backend()
    assert Backend.preset("cuda-fused", device="cuda:1").device == "cuda:1"
    with pytest.raises(ValueError):
        Backend.preset("tpu")


@pytest.mark.parametrize("kw", [dict(kernel="torch"), dict(kernel="nki"),
                                dict(backend=Backend.preset("cpu")), dict(backend=Backend.preset("cuda"))])
def test_kernel_selection_rejects_what_this_package_cannot_run(kw):
    x, y = clouds()
    with pytest.raises(ValueError):
        sinkhorn(x, y, opts=SinkhornOptions(**kw))


def test_rejects_d_over_128():
    with pytest.raises(ValueError):
        S._use_cuda(SinkhornOptions(), 129)


def test_balanced_validation_happens_first():
    x, y = clouds()
    with pytest.raises(ValueError):
        sinkhorn(x, y, a=np.full(len(x), 2.0 / len(x)))
    with pytest.raises(ValueError):
        sinkhorn(x, y, a_target=np.full(len(x), 1.0 / len(x)))
    with pytest.raises(ValueError):
        sinkhorn(x, y, a=-np.ones(len(x)))


def test_cloud_layout_pads_to_row_tiles_per_shard():
    x, _ = clouds(n=300, d=7)
    lw = np.full(300, -np.log(300))
    c = S._Cloud(x, lw, shards=2, dev=torch.device("cpu"), off=np.ones(300))
    assert c.npad == 512 and c.xT.shape == (7, 512)
    assert torch.all(c.xT[:, 300:] == 0)
    assert torch.all(c.log_w[300:] == np.float32(S.PAD_LOG_WEIGHT))
    assert torch.all(c.w[300:] == 0) and torch.all(c.off[300:] == 0) and torch.all(c.off[:300] == 1)
    np.testing.assert_allclose(c.sq.numpy()[:300], (x * x).sum(1), rtol=1e-6)


def test_shard_ranges_cover_rows_once():
    for shards in (1, 2, 4, 8):
        npad = 128 * shards * 3
        seen = np.zeros(npad, int)
        for r in range(shards):
            a, b = S._shard_range(npad, shards, r)
            assert a % 128 == 0
            seen[a:b] += 1
        assert np.all(seen == 1)
    with pytest.raises(ValueError):
        S._shard_range(128 * 3, 2, 0)


def _cta_of(u, U, G):          # the kernels' sk_cta_of (csrc/common.cuh)
    return ((u + 1) * G + U - 1) // U - 1


def _begin(k, U, G):
    return (k * U) // G


@pytest.mark.parametrize("U,G", [(1, 1), (7, 3), (6241, 296), (3160, 148), (79, 148), (100, 100), (1000, 7)])
def test_stream_k_split(U, G):
    """Every unit is owned by exactly the CTA sk_cta_of names, and no CTA range is empty when G <= U."""
    G = min(G, U)
    owner = np.empty(U, int)
    for k in range(G):
        a, b = _begin(k, U, G), _begin(k + 1, U, G)
        assert b > a
        owner[a:b] = k
    for u in range(U):
        assert _cta_of(u, U, G) == owner[u]


def test_stream_k_slot_bound():
    """sk_max_slots bounds the number of CTAs that touch one row tile."""
    for nrt, nct, G in [(79, 79, 296), (79, 40, 148), (3, 500, 148), (200, 2, 148), (1, 1, 1), (2048, 2048, 148)]:
        U = nrt * nct
        G = min(G, U)
        bound = (nct * G + U - 1) // U + 1
        for r in range(nrt):
            touched = _cta_of(r * nct + nct - 1, U, G) - _cta_of(r * nct, U, G) + 1
            assert touched <= bound


def test_wot_eps_stages_match_oracle():
    from trnopt.singlecell import wot_eps_stages
    for eps in (0.05, 0.2, 0.01):
        assert wot_eps_stages(eps) == O.wot_eps_stages(eps)


def test_synthetic_generators_are_seeded():
    a, b = synthetic.cfg1()
    a2, b2 = synthetic.cfg1()
    assert a.shape == (2000, 16) and np.array_equal(a, a2) and np.array_equal(b, b2)
    x0, x1, g = synthetic.cfg3(n=50, m=60)
    assert x0.shape == (50, 30) and x1.shape == (60, 30) and g.shape == (50,) and np.all(g > 0)
    tr = synthetic.cfg4()
    assert len(tr.cohorts) == 39 and abs(sum(len(c) for c in tr.cohorts) - 175_000) < 100
    stages = synthetic.cfg5_eps_stages()
    assert len(stages) == 7 and stages[0] == 1.0 and abs(stages[-1] / 0.01 - (1 / 0.01) ** (1 / 7)) < 1e-9


def test_exchange_selection():
    """cores > 1: peer stores on the tc path by default, the NCCL all-gather on the FFMA path; bad names raise."""
    import trnopt.sinkhorn  # noqa: F401
    S = sys.modules["trnopt.sinkhorn"]
    assert S._exchange("auto", "tc") == "peer"
    assert S._exchange("auto", "ffma") == "nccl"
    assert S._exchange("nccl", "tc") == "nccl"
    with pytest.raises(ValueError):
        S._exchange("peer", "ffma")
    with pytest.raises(ValueError):
        S._exchange("mpi", "tc")
