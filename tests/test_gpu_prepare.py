"""The solve's device-side set-up and tear-down (trnopt_cloud_stats, trnopt_prepare_cloud, trnopt_unshift,
trnopt_take_error_flags) against host float64 arithmetic and against the torch-built layout of _Cloud, and the
buffers kept between solves of one shape."""

import numpy as np
import pytest
import torch

import trnopt.sinkhorn  # noqa: F401  (the module; the package attribute of that name is the function)
from trnopt import Backend, SinkhornOptions, _capi, sinkhorn

pytestmark = pytest.mark.gpu
S = __import__("sys").modules["trnopt.sinkhorn"]


def _clouds(n=1000, m=1500, d=30, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(size=(n, d)) * 3 + 1, rng.uniform(-2, 5, size=(m, d))


def test_cloud_stats_match_numpy():
    x, y = _clouds()
    xd, yd = torch.as_tensor(x).cuda(), torch.as_tensor(y).cuda()
    st = torch.empty((2, 3, x.shape[1]), dtype=torch.float64, device="cuda")
    scratch = _capi.cloud_stats_scratch(x.shape[1], "cuda")
    for _ in range(2):                                   # the scratch is left ready for the next call
        _capi.cloud_stats(xd, yd, st, scratch)
        h = st.cpu().numpy()
        for c, p in enumerate((x, y)):
            np.testing.assert_allclose(h[c, 0], p.sum(0), rtol=1e-13, atol=1e-12)
            np.testing.assert_array_equal(h[c, 1], p.min(0))
            np.testing.assert_array_equal(h[c, 2], p.max(0))


@pytest.mark.parametrize("path", ["tc", "ffma"])
def test_prepare_cloud_matches_the_torch_layout(path):
    """Same padded layout as _Cloud built with torch ops on the device: float64 norms to rounding, float32 vectors,
    the FP16 [hi | lo] rows bit for bit (the same float32 coordinates split the same way), the initial potential."""
    d = 30 if path == "tc" else 70
    x, y = _clouds(d=d)
    n = len(x)
    rng = np.random.default_rng(3)
    lw = np.log(rng.uniform(0.5, 1.5, n) / n)
    off = rng.normal(scale=0.2, size=n)
    center, r = np.full(d, 0.3), 1.7
    xs = (x - center) / r
    shift = (xs.sum(0) + ((y - center) / r).sum(0)) / (n + len(y))
    xi = xs - shift
    ref = S._Cloud(torch.as_tensor(xi).cuda(), lw, 2, torch.device("cuda"), off)
    ref.sexp = S._scale_exp(np.abs(xi).max())
    if path == "tc":
        ref.pack()
    dc = S._DeviceCloud(n, d, 2, torch.device("cuda"), path)
    dc.upload(x, lw, False, off)
    dc.sexp = ref.sexp
    gh0 = torch.empty(dc.npad, dtype=torch.float32, device="cuda")
    dc.prepare(center, r, shift, 0.0, gh0=gh0)
    torch.cuda.synchronize()
    assert dc.npad == ref.npad
    np.testing.assert_allclose(dc.sq64.cpu().numpy(), ref.sq64.cpu().numpy(), rtol=1e-14, atol=1e-14)
    for a, b in ((dc.log_w, ref.log_w), (dc.off, ref.off)):
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    np.testing.assert_allclose(dc.w.cpu().numpy(), ref.w.cpu().numpy(), rtol=1e-7)
    np.testing.assert_allclose(dc.sq.cpu().numpy(), ref.sq.cpu().numpy(), rtol=1e-7)
    if path == "tc":
        np.testing.assert_array_equal(dc.packed.view(torch.int16).cpu().numpy(),
                                      ref.packed.view(torch.int16).cpu().numpy())
    else:
        np.testing.assert_array_equal(dc.xT.cpu().numpy(), ref.xT.cpu().numpy())
    g0 = (xs * xs).sum(1) - (xi * xi).sum(1)
    np.testing.assert_allclose(gh0.cpu().numpy()[:n], g0, rtol=1e-6, atol=1e-6)
    assert not gh0.cpu().numpy()[n:].any()


def test_unshift_and_error_flags_in_one_download():
    h = torch.linspace(-3, 3, 1000, device="cuda")
    sq = torch.rand(1000, dtype=torch.float64, device="cuda")
    out = torch.full((1002,), np.nan, dtype=torch.float64, device="cuda")
    _capi.unshift(h, sq, 1000, out)
    _capi.take_error_flags(S._Off(out, 1001, 8))
    o = out.cpu().numpy()
    np.testing.assert_array_equal(o[:1000], h.double().cpu().numpy() + sq.cpu().numpy())
    assert np.isnan(o[1000]) and o[1001] == 0.0


def test_buffers_are_reused_between_solves_of_one_shape():
    """Solves of shape A, then B, then A again (and A with other weights) on one thread: the kept buffers give the
    same answers as fresh ones, bit for bit."""
    be = Backend.preset("cuda-fused")
    o = SinkhornOptions(eps=0.1, max_iters=15, fixed_iters=True, normalize=False, backend=be)
    xa, ya = _clouds(300, 260, 16, 1)
    xb, yb = _clouds(500, 410, 16, 2)
    r1 = sinkhorn(xa, ya, opts=o)
    sinkhorn(xb, yb, opts=o)
    r2 = sinkhorn(xa, ya, opts=o)
    np.testing.assert_array_equal(r1.f, r2.f)
    np.testing.assert_array_equal(r1.g, r2.g)
    wa = np.random.default_rng(0).uniform(0.5, 1.5, 300)
    wa /= wa.sum()
    rw = sinkhorn(xa, ya, wa, None, o)
    S._Buffers._cache.clear()
    rw2 = sinkhorn(xa, ya, wa, None, o)
    np.testing.assert_array_equal(rw.f, rw2.f)
    assert np.abs(rw.f - r1.f).max() > 1e-6
