"""Data-parallel plumbing: one process per GPU, NCCL communicator owned by
libtpcuda, bootstrapped through the ranks' own file store (tpcuda.store),
which hands the NCCL unique id from rank 0 to the other ranks.
"""
from __future__ import annotations

import ctypes
import os

from ._lib import check
from .store import FileStore

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

    def check_peers(self, store: FileStore) -> None:
        """Between steps: raise if a rank has left (FileStore.leave), before any
        collective is issued that would wait for it."""
        gone = store.departed()
        if gone:
            raise RuntimeError(f"rank(s) {gone} left the job; no further collective is issued")

    def world_now(self) -> int:
        r, w = ctypes.c_int(0), ctypes.c_int(0)
        check(self.lib.tp_comm_info(ctypes.byref(r), ctypes.byref(w)))
        return int(w.value)


def env_ranks() -> tuple[int, int, int]:
    """(rank, world, local rank) from the launcher's environment (torchrun's
    RANK / WORLD_SIZE / LOCAL_RANK; a single process when absent)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def comm_from_store(lib, store: FileStore) -> NcclComm | None:
    """Create the NCCL communicator of the store's ranks (None for one rank):
    rank 0 draws the unique id and publishes it, the others wait for it."""
    if store.world == 1:
        return None
    uid = NcclComm.unique_id(lib) if store.rank == 0 else None
    uid = store.broadcast_bytes(uid, "nccl-unique-id")
    return NcclComm(lib, store.rank, store.world, uid)
