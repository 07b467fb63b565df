"""The multi-GPU host logic on CPU with two gloo ranks: every rank computes its shard of rows of a half-step and
the product's in-place all-gather (_gather_rows) assembles the full potential on every rank. The half-step itself is
stood in for by the CPU oracle (the test is of the sharding, not of the kernel). CPU only."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        for p in (ROOT, ROOT / "trainium-sinkhorn_b200"):
            sys.path.insert(0, str(p))
        import trnopt.sinkhorn  # noqa: F401
        from oracle import trnopt_oracle as O
        S = sys.modules["trnopt.sinkhorn"]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(0)
        x, y = rng.normal(size=(300, 6)), rng.normal(size=(211, 6))
        X = S._Cloud(x, np.full(300, -np.log(300)), world, torch.device("cpu"))
        Y = S._Cloud(y, np.full(211, -np.log(211)), world, torch.device("cpu"))
        gh = torch.as_tensor(rng.normal(size=Y.npad), dtype=torch.float32)
        r0, r1 = S._shard_range(X.npad, world, rank)
        out = torch.full((X.npad,), float("nan"))
        xs = X.xT.T.contiguous()
        out[r0:r1] = O.half_step(xs[r0:r1], X.sq[r0:r1], X.off[r0:r1], Y.xT, gh, Y.log_w, 10.0, 0.1, 0.9)
        S._gather_rows(out, r0, r1)
        full = O.half_step(xs, X.sq, X.off, Y.xT, gh, Y.log_w, 10.0, 0.1, 0.9)
        q.put((rank, float((out - full).abs().max()), (r0, r1)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world", [2])
def test_sharded_rows_and_gather(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    ranges = sorted(r[2] for r in res if r[2] is not None)
    for rank, err, rng in res:
        assert rng is not None, err
        assert err == 0.0, (rank, err)
    assert ranges[0][0] == 0 and ranges[0][1] == ranges[1][0]
