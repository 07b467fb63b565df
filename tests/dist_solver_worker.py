"""Worker for tests/test_gpu_multi.py: one rank per GPU (launched by torchrun), solves the same problems with the
rows of every half-step split across the ranks (SinkhornOptions(cores=world)), once with each exchange (peer stores
from the kernels, NCCL all-gather), and rank 0 saves the results."""
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "trainium-sinkhorn_b200")]

import datetime  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from trnopt import Backend, SinkhornOptions, sinkhorn  # noqa: E402


def peer_timeout(out):
    """Rank 1 joins the peer region and then skips its half-steps (a host decision between steps, none of its kernels
    in flight); rank 0's run waits for rank 1's rows, gives up after the kernels' time limit and reports error bit 8
    (another GPU did not publish) through trnopt_device_error_flags."""
    from trnopt import _capi, _comm
    import trnopt.sinkhorn  # noqa: F401
    S = sys.modules["trnopt.sinkhorn"]
    rank = dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(0)
    x, y = rng.uniform(size=(600, 16)), rng.uniform(size=(500, 16))
    X = S._Cloud(x, np.full(600, -np.log(600)), 2, dev)
    Y = S._Cloud(y, np.full(500, -np.log(500)), 2, dev)
    X.pack()
    Y.pack()
    ws = S._workspace(X, Y, 2, dev, "tc")
    reg = _comm.PeerRegion(4 * (X.npad + 2 * Y.npad))
    fh = reg.tensor(0, X.npad)
    G = [reg.tensor(4 * X.npad, Y.npad), reg.tensor(4 * (X.npad + Y.npad), Y.npad)]
    G[0].zero_()
    fh.zero_()
    reg.arrive()
    flags = -1
    if rank == 0:
        _capi.sinkhorn_run_sharded(reg.comm, X.packed, X.sq, None, X.log_w, X.npad, X.sexp, Y.packed, Y.sq, None,
                                   Y.log_w, Y.npad, Y.sexp, X.d, G[0], G[1], fh, 0, 1, 0.1, 1.0, 1.0, ws)
        torch.cuda.synchronize()
        flags = _capi.device_error_flags()
        np.savez(out, flags=flags)
    dist.barrier()


def main():
    out = sys.argv[1]
    if len(sys.argv) > 2 and sys.argv[2] == "peer_timeout":
        local = int(os.environ["LOCAL_RANK"])
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=60))
        peer_timeout(out)
        dist.destroy_process_group()
        return
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=60))
    world = dist.get_world_size()
    be = Backend.preset("cuda-fused", device=f"cuda:{local}")
    res = {"world": world}
    # Both exchanges, three solves each: the second reuses the peer region, the third needs a larger one.
    for ex in ("peer", "nccl"):
        rng = np.random.default_rng(0)
        x, y = rng.uniform(size=(1500, 16)), rng.uniform(size=(1300, 16))
        r = sinkhorn(x, y, opts=SinkhornOptions(eps=0.1, max_iters=60, fixed_iters=True, normalize=False, cores=world,
                                                backend=be, cuda_exchange=ex))
        xu, yu = rng.uniform(size=(700, 8)), rng.uniform(size=(650, 8))
        a = rng.uniform(0.5, 1.5, 700) / 700
        ru = sinkhorn(xu, yu, a=a, opts=SinkhornOptions(eps=0.1, rho=1.0, tol=1e-5, max_iters=3000, cores=world,
                                                        backend=be, cuda_exchange=ex))
        xb, yb = rng.uniform(size=(5000, 32)), rng.uniform(size=(4100, 32))
        rb = sinkhorn(xb, yb, opts=SinkhornOptions(eps=0.05, tol=1e-5, max_iters=2000, normalize=False, cores=world,
                                                   backend=be, cuda_exchange=ex))
        res.update({f"{ex}_f": r.f, f"{ex}_g": r.g, f"{ex}_fu": ru.f, f"{ex}_gu": ru.g,
                    f"{ex}_row_mass": ru.row_mass, f"{ex}_iters": ru.iterations, f"{ex}_fb": rb.f, f"{ex}_gb": rb.g,
                    f"{ex}_iters_b": rb.iterations})
    if dist.get_rank() == 0:
        np.savez(out, **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
