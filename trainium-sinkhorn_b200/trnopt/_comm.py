"""Peer-mapped device regions for the sharded solver (the trnopt_comm_* entries of the C ABI).

Every rank of a process group (one process per GPU) allocates one region, the ranks exchange CUDA IPC handles through
the group, and each maps the others' regions. The solver keeps the gathered potentials (fh and the two g buffers) in
the region, so a half-step can store its rows straight into every GPU's copy (trnopt_sinkhorn_run_sharded) instead
of following each half-step with an all-gather. Creating, growing and closing a region are collective: every rank
of the group must make the same calls in the same order, as it does for any collective.
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi
from ._capi import check, lib

MAX_RANKS = 8


class _Cai:
    """A float32 vector in device memory, handed to torch.as_tensor through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2,
                                         "strides": None}


class PeerRegion:
    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"peer regions support at most {MAX_RANKS} ranks")
        self.dev = torch.device("cuda", torch.cuda.current_device())
        hb = int(lib.trnopt_comm_handle_bytes())
        handle = ctypes.create_string_buffer(hb)
        comm = ctypes.c_void_p()
        check(lib.trnopt_comm_create(self.rank, self.world, int(nbytes), ctypes.byref(comm), handle),
              "trnopt_comm_create")
        self.comm = comm
        on_dev = dist.get_backend(group) == "nccl"
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8)
        mine = mine.to(self.dev) if on_dev else mine
        every = torch.empty(self.world * hb, dtype=torch.uint8, device=mine.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        check(lib.trnopt_comm_open(comm, bytes(every.cpu().numpy())), "trnopt_comm_open")
        self.base = int(lib.trnopt_comm_buffer(comm))
        self.nbytes = int(lib.trnopt_comm_buffer_bytes(comm))

    def tensor(self, offset_bytes: int, n: int) -> torch.Tensor:
        """n float32 values at offset_bytes into this rank's buffer (the same offset on every rank)."""
        if offset_bytes % 4 or offset_bytes + 4 * n > self.nbytes:
            raise ValueError("view outside the region")
        return torch.as_tensor(_Cai(self.base + offset_bytes, n), device=self.dev)

    def arrive(self) -> None:
        check(lib.trnopt_comm_arrive(self.comm, _capi._stream()), "trnopt_comm_arrive")

    def wait(self) -> None:
        check(lib.trnopt_comm_wait(self.comm, _capi._stream()), "trnopt_comm_wait")

    def close(self) -> None:
        """Collective: every rank synchronises, meets the others, then unmaps and frees."""
        import torch.distributed as dist
        if self.comm is None:
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        check(lib.trnopt_comm_destroy(self.comm), "trnopt_comm_destroy")
        self.comm = None


_REGIONS: dict = {}


def region(nbytes: int, group=None) -> PeerRegion:
    """The process's region for `group` on the current device, created or grown (collectively) to nbytes. The
    default group is resolved to the process group object itself, so a re-initialised default group (with possibly
    another world size) gets its own region rather than one mapped for the previous group's ranks."""
    import torch.distributed as dist
    g = group if group is not None else dist.group.WORLD
    key = (id(g), torch.cuda.current_device())
    r = _REGIONS.get(key)
    if r is not None and r.group_obj is not g:      # the id of a dead group reused by a new object
        r = None
    if r is not None and r.nbytes >= nbytes:
        return r
    if r is not None:
        r.close()
        nbytes = max(nbytes, 2 * r.nbytes)
    r = _REGIONS[key] = PeerRegion(nbytes, group)
    r.group_obj = g
    return r
