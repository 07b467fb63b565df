"""Worker for tests/test_gpu_multi.py: one rank per GPU (launched by torchrun), solves the same problem with the
rows of every half-step split across the ranks (SinkhornOptions(cores=world)) and rank 0 saves the result."""
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
    rng = np.random.default_rng(0)
    x, y = rng.uniform(size=(1500, 16)), rng.uniform(size=(1300, 16))
    be = Backend.preset("cuda-fused", device=f"cuda:{local}")
    r = sinkhorn(x, y, opts=SinkhornOptions(eps=0.1, max_iters=60, fixed_iters=True, normalize=False, cores=world,
                                            backend=be))
    xu, yu = rng.uniform(size=(700, 8)), rng.uniform(size=(650, 8))
    a = rng.uniform(0.5, 1.5, 700) / 700
    ru = sinkhorn(xu, yu, a=a, opts=SinkhornOptions(eps=0.1, rho=1.0, tol=1e-5, max_iters=3000, cores=world,
                                                    backend=be))
    if dist.get_rank() == 0:
        np.savez(out, f=r.f, g=r.g, fu=ru.f, gu=ru.g, row_mass=ru.row_mass, iters=ru.iterations, world=world)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
