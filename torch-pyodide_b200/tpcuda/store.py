"""Host-side rendezvous for the data-parallel ranks of one node.

The NCCL communicator (csrc/tp_comm.cu) needs its unique id handed from rank 0
to every other rank before ``ncclCommInitRank``; the benchmark and the tests
also need barriers and a max over ranks of a timing.  The reference package
has no parallelism at all, and in a process where ``torch`` is the reference
package itself there is no ``torch.distributed`` to borrow, so this module is
the bootstrap: a directory shared by the ranks of one job, where each value is
a file written atomically (write to a temporary name, then rename).

The directory is named from the launcher's environment so that all ranks of
one launch agree on it and two launches never share it: ``TPCUDA_STORE_DIR``
when set, else ``<tmp>/tpcuda-store-<MASTER_PORT>-<parent pid>`` (torchrun's
agent is the parent of every local rank, and its pid is unique while the job
runs).  Every wait is bounded; a rank that never arrives makes the others
raise ``TimeoutError`` instead of hanging.
"""
from __future__ import annotations

import json
import os
import shutil
import tempfile
import time

import numpy as np


def default_dir() -> str:
    d = os.environ.get("TPCUDA_STORE_DIR")
    if d:
        return d
    port = os.environ.get("MASTER_PORT", "0")
    return os.path.join(tempfile.gettempdir(), f"tpcuda-store-{port}-{os.getppid()}")


class FileStore:
    """Key/value store, barrier and all-gather over a shared directory."""

    def __init__(self, rank: int, world: int, path: str | None = None, timeout_s: float = 300.0):
        self.rank, self.world = int(rank), int(world)
        self.path = path or default_dir()
        self.timeout_s = float(timeout_s)
        self._round = 0
        os.makedirs(self.path, exist_ok=True)

    # ---- key / value ----------------------------------------------------------
    def _file(self, key: str) -> str:
        return os.path.join(self.path, key.replace("/", "_"))

    def set(self, key: str, value: bytes) -> None:
        fd, tmp = tempfile.mkstemp(dir=self.path, prefix=".tmp-")
        with os.fdopen(fd, "wb") as f:
            f.write(value)
        os.replace(tmp, self._file(key))

    def get(self, key: str, timeout_s: float | None = None) -> bytes:
        """Wait (bounded) for ``key`` and return its bytes."""
        limit = self.timeout_s if timeout_s is None else float(timeout_s)
        t0 = time.monotonic()
        f = self._file(key)
        delay = 1e-4
        while not os.path.exists(f):
            if time.monotonic() - t0 > limit:
                raise TimeoutError(f"rank {self.rank}: no value for {key!r} after {limit:.0f} s in {self.path}")
            time.sleep(delay)
            delay = min(delay * 2, 0.01)
        with open(f, "rb") as fh:
            return fh.read()

    # ---- collectives on the host ------------------------------------------------
    def all_gather_bytes(self, value: bytes, tag: str = "ag") -> list[bytes]:
        r = self._round
        self._round += 1
        self.set(f"{tag}.{r}.{self.rank}", value)
        return [self.get(f"{tag}.{r}.{k}") for k in range(self.world)]

    def barrier(self) -> None:
        self.all_gather_bytes(b"", "barrier")

    def all_gather_obj(self, obj) -> list:
        return [json.loads(b) for b in self.all_gather_bytes(json.dumps(obj).encode(), "obj")]

    def max(self, value: float) -> float:
        return max(float(v) for v in self.all_gather_obj(float(value)))

    def all_gather_array(self, arr: np.ndarray) -> list[np.ndarray]:
        a = np.ascontiguousarray(arr)
        head = json.dumps({"dtype": a.dtype.str, "shape": list(a.shape)}).encode()
        blobs = self.all_gather_bytes(len(head).to_bytes(4, "little") + head + a.tobytes(), "arr")
        out = []
        for b in blobs:
            n = int.from_bytes(b[:4], "little")
            meta = json.loads(b[4:4 + n])
            out.append(np.frombuffer(b[4 + n:], dtype=np.dtype(meta["dtype"])).reshape(meta["shape"]).copy())
        return out

    def broadcast_bytes(self, value: bytes | None, key: str, src: int = 0) -> bytes:
        if self.rank == src:
            self.set(key, value)
            return value
        return self.get(key)

    # ---- departures ---------------------------------------------------------
    def leave(self) -> None:
        """Mark this rank as gone, between steps, before it exits early; the
        others see it with ``departed()`` before their next collective instead
        of launching one that would wait for this rank."""
        self.set(f"left.{self.rank}", b"")

    def departed(self) -> list[int]:
        return [k for k in range(self.world) if k != self.rank and os.path.exists(self._file(f"left.{k}"))]

    def close(self) -> None:
        """Every rank leaves a last mark and reads nothing after it; rank 0
        waits for all marks, then removes the directory."""
        self.set(f"closed.{self.rank}", b"")
        if self.rank == 0:
            for k in range(self.world):
                self.get(f"closed.{k}")
            shutil.rmtree(self.path, ignore_errors=True)
