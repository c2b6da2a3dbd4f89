"""Input pipeline host logic on the CPU.

* tpcuda.data.PinnedLoader over a fake runtime whose "pinned" buffers are host
  memory and whose async upload copies at once: batch order, shuffling (one
  numpy permutation per epoch), drop_last, dtype coercion (integer tags
  truncate, bool is 0/1), the staging ring (a slot is refilled only after its
  previous copy's ticket was waited on, and every batch's ticket is marked used
  before the batch is handed out).
* The patched reference DataLoader over a TensorDataset yields the same batches,
  in the same sampler order, as the reference's per-sample path (oracle).
"""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from tpcuda.data import PinnedLoader

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


class FakeRT:
    def __init__(self):
        self.bufs, self.events, self.next_ticket = {}, [], 1
        self.done = set()

    def hostAlloc(self, n):
        b = ctypes.create_string_buffer(n)
        p = ctypes.addressof(b)
        self.bufs[p] = b
        return p

    def hostFree(self, p):
        self.bufs.pop(p)

    def tensorFromHostAsync(self, ptr, shape, dtype, defer=False):
        n = int(np.prod(shape))
        arr = np.ctypeslib.as_array(ctypes.cast(ctypes.c_void_p(ptr), ctypes.POINTER(ctypes.c_float)), (n,)).copy()
        t = self.next_ticket
        self.next_ticket += 1
        self.events.append(("upload", t, ptr))
        return {"data": arr.reshape(shape), "dtype": dtype, "shape": list(shape)}, t

    def ticketUse(self, t):
        self.events.append(("use", t))

    def ticketWait(self, t):
        self.events.append(("wait", t))


@pytest.mark.parametrize("shuffle,drop_last,depth", [(False, False, 2), (True, False, 2), (True, True, 3),
                                                     (False, True, 1)])
def test_pinned_loader_batches(shuffle, drop_last, depth):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((23, 3, 4)).astype(np.float32)
    y = rng.integers(-5, 10, 23).astype(np.int64)
    m = rng.integers(0, 2, 23).astype(bool)
    rt = FakeRT()
    ld = PinnedLoader(rt, [x, y, m], batch_size=5, shuffle=shuffle, drop_last=drop_last,
                      dtypes=["float32", "int64", "bool"], seed=7, depth=depth)
    order = np.random.default_rng(7).permutation(23) if shuffle else np.arange(23)
    want = [order[i:i + 5] for i in range(0, 23, 5)]
    if drop_last:
        want = [w for w in want if len(w) == 5]
    got = list(ld)
    assert len(got) == len(want) == len(ld)
    for (bx, by, bm), idx in zip(got, want):
        assert np.array_equal(bx["data"], x[idx])
        assert np.array_equal(by["data"], np.trunc(y[idx].astype(np.float64)).astype(np.float32))
        assert np.array_equal(bm["data"], m[idx].astype(np.float32))
        assert by["dtype"] == "int64" and bm["dtype"] == "bool"
    # every upload's ticket is marked used before its batch is handed out, and a
    # staging buffer is refilled only after the copy that last used it was waited on
    uploads = [e for e in rt.events if e[0] == "upload"]
    last_on_ptr = {}
    for i, e in enumerate(rt.events):
        if e[0] == "upload":
            prev = last_on_ptr.get(e[2])
            if prev is not None:
                assert ("wait", prev) in rt.events[:i]
            last_on_ptr[e[2]] = e[1]
    used = [e[1] for e in rt.events if e[0] == "use"]
    assert sorted(used) == [u[1] for u in uploads]
    ld.close()
    assert not rt.bufs


DL_SCRIPT = r"""
import sys, json, random
import numpy as np
sys.path[:0] = [{pkg!r}, {orc!r}]
from tpcuda import shim, patches
from oracle_runtime import OracleRuntime
rt = OracleRuntime(); shim.install(rt)
sys.path.insert(0, {ref!r})
import torch
from torch.utils.data import DataLoader, TensorDataset
if {patched}:
    patches.apply()
rng = np.random.default_rng(1)
x = torch.tensor(rng.standard_normal((11, 2, 3)).astype(np.float32).tolist())
y = torch.tensor(rng.integers(0, 4, 11).tolist(), dtype=torch.int64)
random.seed(5)
out = []
for bx, by in DataLoader(TensorDataset(x, y), batch_size=4, shuffle=True):
    out.append([bx.tolist(), by.tolist(), list(bx.shape), by.dtype])
print(json.dumps(out))
"""


def test_patched_dataloader_matches_reference_batches():
    sys.path.insert(0, HERE)
    from dropin_train import reference_path
    ref = reference_path()
    if ref is None:
        pytest.skip("reference package not installed (baseline/_ref)")
    outs = []
    for patched in (False, True):
        code = DL_SCRIPT.format(pkg=os.path.join(ROOT, "torch-pyodide_b200"), orc=os.path.join(ROOT, "oracle"),
                                ref=ref, patched=patched)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-3000:]
        outs.append(json.loads(r.stdout.strip().splitlines()[-1]))
    assert outs[0] == outs[1] and len(outs[0]) == 3
