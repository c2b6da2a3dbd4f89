"""Input pipeline: host datasets to HBM batches without Python lists.

The reference's data path builds every batch on the host as Python lists:
``DataLoader`` indexes a ``TensorDataset`` one sample at a time and stacks the
samples (python/torch/utils/data/__init__.py:24-37,205-210), and
``torch.tensor(data)`` flattens its data to a list before ``tensorFromData``
(python/torch/tensor_factories_ops.py:18-25).

``PinnedLoader`` serves datasets held in host memory as numpy arrays (images,
labels, ...): each batch is gathered with numpy straight into a pinned staging
buffer and uploaded with ``tensorFromHostAsync``, which runs on the library's
copy stream, so the upload of batch i+1 overlaps the kernels of batch i; the
library's compute stream is made to wait for a batch's copy just before the
batch is handed out.  A
ring of ``depth`` staging slots is reused; before a slot is refilled its
previous upload's ticket is waited on.  Values take the runtime's storage
convention: float32 whatever the dtype tag, integer tags truncated toward zero,
bool as 0/1 (runtime/src/ops/creationOps.ts:25-37).

For a dataset already on the device (a reference ``TensorDataset``),
``tpcuda.patches`` makes the reference ``DataLoader`` gather each batch with
one ``gatherRows`` call instead.
"""
from __future__ import annotations

import ctypes

import numpy as np


def _coerce(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bool":
        return (a != 0).astype(np.float32)
    if dtype.startswith("uint"):
        return np.maximum(np.trunc(a.astype(np.float64)), 0).astype(np.float32)
    if dtype.startswith("int"):
        return np.trunc(a.astype(np.float64)).astype(np.float32)
    return np.asarray(a, np.float32)


class _Slot:
    def __init__(self, rt, nbytes: int):
        self.rt = rt
        self.ptr = rt.hostAlloc(nbytes)
        self.nbytes = nbytes
        self.view = np.ctypeslib.as_array(ctypes.cast(ctypes.c_void_p(self.ptr), ctypes.POINTER(ctypes.c_float)),
                                          shape=(nbytes // 4,))
        self.ticket = 0

    def free(self):
        if self.ptr:
            if self.ticket:
                self.rt.ticketWait(self.ticket)
            self.rt.hostFree(self.ptr)
            self.ptr = 0


class PinnedLoader:
    """Batches of host arrays, delivered as device tensors.

    arrays: numpy arrays sharing their first dimension (samples);
    dtypes: the runtime dtype tag of each (default "float32"); batch_size,
    shuffle, drop_last: as the reference ``DataLoader``; seed: the shuffle's
    numpy seed (one permutation per epoch); depth: staging slots in flight;
    wrap: turns a runtime handle dict into what the loader yields (e.g. a
    reference ``torch.Tensor``; default: the handle dict itself)."""

    def __init__(self, rt, arrays, batch_size: int, shuffle: bool = False, drop_last: bool = False,
                 dtypes=None, seed: int = 0, depth: int = 2, wrap=None):
        self.rt = rt
        self.arrays = [np.asarray(a) for a in arrays]
        n = self.arrays[0].shape[0]
        if any(a.shape[0] != n for a in self.arrays):
            raise ValueError("PinnedLoader: arrays must share their first dimension")
        self.n = n
        self.batch_size = int(batch_size)
        self.shuffle, self.drop_last = bool(shuffle), bool(drop_last)
        self.dtypes = list(dtypes) if dtypes is not None else ["float32"] * len(self.arrays)
        self.rng = np.random.default_rng(seed)
        self.depth = max(1, int(depth))
        self.wrap = wrap or (lambda h: h)
        self.row = [int(np.prod(a.shape[1:], dtype=np.int64)) for a in self.arrays]
        self.slots = [[_Slot(rt, max(16, self.batch_size * r * 4)) for r in self.row] for _ in range(self.depth)]
        self._k = 0

    def __len__(self) -> int:
        return self.n // self.batch_size if self.drop_last else -(-self.n // self.batch_size)

    def batches(self):
        """The index lists of one epoch, in order (the reference's BatchSampler)."""
        order = self.rng.permutation(self.n) if self.shuffle else np.arange(self.n)
        out = [order[i:i + self.batch_size] for i in range(0, self.n, self.batch_size)]
        if self.drop_last and out and len(out[-1]) < self.batch_size:
            out.pop()
        return out

    def _upload(self, idx):
        slots = self.slots[self._k % self.depth]
        self._k += 1
        handles = []
        for a, dt, r, slot in zip(self.arrays, self.dtypes, self.row, slots):
            if slot.ticket:
                self.rt.ticketWait(slot.ticket)  # the slot's previous copy has left the buffer
            k = len(idx)
            dst = slot.view[:k * r].reshape((k,) + a.shape[1:])
            dst[...] = _coerce(np.take(a, idx, axis=0), dt)
            h, slot.ticket = self.rt.tensorFromHostAsync(slot.ptr, [k] + list(a.shape[1:]), dt, defer=True)
            handles.append((h, slot.ticket))
        return handles

    def __iter__(self):
        todo = self.batches()
        pending = [self._upload(b) for b in todo[:self.depth]]
        for i in range(len(todo)):
            cur = pending.pop(0)
            if i + self.depth < len(todo):
                # staged while batch i is consumed; this slot's last copy (batch
                # i + depth - depth = i) must be finished first: ticketWait
                pending.append(self._upload(todo[i + self.depth]))
            for _, tk in cur:  # kernels issued from here on see this batch's copy
                self.rt.ticketUse(tk)
            yield tuple(self.wrap(h) for h, _ in cur)

    def close(self):
        for slots in self.slots:
            for s in slots:
                s.free()
        self.slots = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
