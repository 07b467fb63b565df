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


def main():
    out = sys.argv[1]
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
