"""Rows of every half-step split across 2 or 4 GPUs (one process per GPU; the new potential reaches every GPU either by
peer stores from the half-step kernels or by an NCCL all-gather) give the single-GPU answer: the counterpart of the
reference's two-cores-match-one test (tests/test_sinkhorn.py:174-183)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4])
def test_gpus_match_one(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from trnopt import Backend, SinkhornOptions, sinkhorn
    out = tmp_path / f"world{world}.npz"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "420", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29600 + world + os.getpid() % 200}",
           str(ROOT / "tests" / "dist_solver_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    z = np.load(out)
    rng = np.random.default_rng(0)
    x, y = rng.uniform(size=(1500, 16)), rng.uniform(size=(1300, 16))
    be = Backend.preset("cuda-fused")
    one = sinkhorn(x, y, opts=SinkhornOptions(eps=0.1, max_iters=60, fixed_iters=True, normalize=False, backend=be))
    xu, yu = rng.uniform(size=(700, 8)), rng.uniform(size=(650, 8))
    a = rng.uniform(0.5, 1.5, 700) / 700
    ru = sinkhorn(xu, yu, a=a, opts=SinkhornOptions(eps=0.1, rho=1.0, tol=1e-5, max_iters=3000, backend=be))
    xb, yb = rng.uniform(size=(5000, 32)), rng.uniform(size=(4100, 32))
    rb = sinkhorn(xb, yb, opts=SinkhornOptions(eps=0.05, tol=1e-5, max_iters=2000, normalize=False, backend=be))
    for ex in ("peer", "nccl"):
        np.testing.assert_allclose(z[f"{ex}_f"], one.f, atol=1e-5 * 0.1, err_msg=ex)
        np.testing.assert_allclose(z[f"{ex}_g"], one.g, atol=1e-5 * 0.1, err_msg=ex)
        assert int(z[f"{ex}_iters"]) == ru.iterations, ex
        np.testing.assert_allclose(z[f"{ex}_fu"], ru.f, atol=1e-5, err_msg=ex)
        np.testing.assert_allclose(z[f"{ex}_row_mass"], ru.row_mass, rtol=1e-4, err_msg=ex)
        assert abs(int(z[f"{ex}_iters_b"]) - rb.iterations) <= 10, ex
        np.testing.assert_allclose(z[f"{ex}_fb"], rb.f, atol=2e-4, err_msg=ex)   # |f| ~ 10: 2e-5 relative
    # the two exchanges move the same float32 rows: identical results
    for k in ("f", "g", "fu", "gu", "fb", "gb"):
        np.testing.assert_array_equal(z[f"peer_{k}"], z[f"nccl_{k}"], err_msg=k)


def test_peer_wait_gives_up_when_a_gpu_stops_publishing(tmp_path):
    """Failure detection on the peer exchange without a GPU fault: one rank stops between steps; the other rank's
    half-step waits for its rows, gives up after the kernels' time limit (4 s) and the host reads error bit 8."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "timeout.npz"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={29700 + os.getpid() % 200}",
           str(ROOT / "tests" / "dist_solver_worker.py"), str(out), "peer_timeout"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert int(np.load(out)["flags"]) & 8
