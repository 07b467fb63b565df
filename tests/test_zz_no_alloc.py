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


def _graph_nodes(g) -> int:
    """Nodes of a captured torch CUDA graph (kept with keep_graph=True), counted by the CUDA runtime's
    cudaGraphGetNodes through the runtime library torch has loaded."""
    import ctypes
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaGraphGetNodes.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]
    rt.cudaGraphGetNodes.restype = ctypes.c_int
    n = ctypes.c_size_t(0)
    assert rt.cudaGraphGetNodes(ctypes.c_void_p(g.raw_cuda_graph()), None, ctypes.byref(n)) == 0
    return n.value


def _scale(a):
    return 14 - int(np.ceil(np.log2(np.abs(a).max())))


def _case(rows, m, d, seed):
    """Packed clouds and vectors of one half-step, and its answer from the workspace entry (own workspace)."""
    x, y, gh, lb, off = _problem(rows, m, d, seed)
    xT, ldx = _capi._pad_ld(_dev(x.T))
    yT, ldy = _capi._pad_ld(_dev(y.T))
    sx, sy = _scale(x), _scale(y)
    xp, yp = _capi.pack_cloud(xT, ldx, rows, d, sx), _capi.pack_cloud(yT, ldy, m, d, sy)
    args = (xp, _dev((x * x).sum(1)), _dev(off), yp, _dev(gh), _dev(lb), rows, m, d, sx, sy, 0.1, 0.9)
    ref = torch.empty(rows, device="cuda")
    ws = _capi.new_workspace(_capi.workspace_size(rows, m, d, _capi.PATH_TC), "cuda")
    _capi.half_step_tc(*args, ref, ws)
    return args, ref


def test_static_scratch_matches_workspace_entry_on_two_calls():
    """Two calls in a row of each of two shapes with different row-tile counts (24 and 55 tiles, like the f and g
    half-steps of one solve), alternating, all through the one static array: each call's counters and partials
    start where the previous call of the other shape left them."""
    d = 64
    cases = [_case(3000, 7000, d, 11), _case(7000, 3000, d, 12)]
    for args, _ in cases:
        assert _capi.workspace_size(args[6], args[7], d, _capi.PATH_TC) <= _capi.lib.trnopt_static_scratch_bytes()
    for k in range(4):
        args, ref = cases[k % 2]
        out = torch.full((args[6],), float("nan"), device="cuda")
        _capi.half_step_tc_static(*args, out)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item() / 0.1
        assert np.isfinite(out.cpu().numpy()).all() and err <= HS_TOL, (k, err)
    assert _capi.device_error_flags() == 0


def test_static_scratch_covers_100k_squared_on_this_gpu():
    """The limit stated in the header: a 100,000^2 (d 64) half-step fits the static array on this device (the need
    depends on the SM count through the stream-K split)."""
    assert _capi.workspace_size(100_000, 100_000, 64, _capi.PATH_TC) <= _capi.lib.trnopt_static_scratch_bytes()


def test_static_scratch_rejects_problems_over_the_limit():
    # 262,144^2 at d 64 needs about 8 MB of partials: more than the 4 MiB array. Rejected before any launch.
    rows = m = 262_144
    assert _capi.workspace_size(rows, m, 64, _capi.PATH_TC) > _capi.lib.trnopt_static_scratch_bytes()
    t = torch.zeros(256, device="cuda")
    with pytest.raises(_capi.TrnoptError, match="static array"):
        _capi.half_step_tc_static(t, t, None, t, t, t, rows, m, 64, 0, 0, 0.1, 1.0, t)


def test_static_scratch_rejected_call_enqueues_nothing():
    """A call that fails an argument check (here eps = 0) returns its status before touching the stream: recorded
    inside a graph capture, it leaves the captured graph empty."""
    t = torch.zeros(256, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.stream(s):
        g.capture_begin(capture_error_mode="thread_local")
        try:
            with pytest.raises(_capi.TrnoptError, match="invalid argument"):
                _capi.half_step_tc_static(t, t, None, t, t, t, 128, 256, 64, 0, 0, 0.0, 1.0, t)
        finally:
            g.capture_end()
    assert _graph_nodes(g) == 0
