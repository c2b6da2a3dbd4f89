"""Data-parallel plumbing: one process per GPU, NCCL communicator owned by
libtpcuda, bootstrapped through torch.distributed (used only to hand the NCCL
unique id from rank 0 to the other ranks and for barriers / timing maxima).
"""
from __future__ import annotations

import ctypes

from ._lib import check

UID_BYTES = 128


class NcclComm:
    """In-place gradient all-reduce on libtpcuda's communication stream."""

    def __init__(self, lib, rank: int, world: int, uid: bytes):
        self.lib, self.rank, self.world = lib, rank, world
        check(lib.tp_comm_init(rank, world, uid, len(uid)))

    @staticmethod
    def unique_id(lib) -> bytes:
        buf = ctypes.create_string_buffer(UID_BYTES)
        check(lib.tp_comm_unique_id(buf, UID_BYTES))
        return buf.raw

    def allreduce_async(self, ptr: int, count: int) -> None:
        check(self.lib.tp_comm_allreduce_async(ctypes.c_void_p(ptr), int(count)))

    def wait(self) -> None:
        check(self.lib.tp_comm_wait())

    def sync(self, timeout_ms: int = 60000) -> None:
        check(self.lib.tp_comm_sync(int(timeout_ms)))

    def close(self) -> None:
        check(self.lib.tp_comm_destroy())


def comm_from_torch_dist(lib) -> NcclComm | None:
    """Create the NCCL communicator for the current torch.distributed group
    (None for a single process)."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return None
    rank, world = dist.get_rank(), dist.get_world_size()
    obj = [NcclComm.unique_id(lib) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return NcclComm(lib, rank, world, obj[0])
