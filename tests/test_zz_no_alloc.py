"""The allocation-free cross-entropy mean (tpk_cross_entropy_mean_noalloc).

Some callers cannot allocate device memory once they are running: a serving
process that reserves its whole HBM budget at start-up, or a latency-critical
loop where an allocation could block or fail.  This entry point gives them the
mean cross-entropy loss using only the inputs and the one-float output they
pass, with its working memory in a fixed array inside the library.  The test
checks it through the C ABI against the allocating entry
(tpk_cross_entropy_mean) on different batches called back to back, so a later
call cannot pass by reusing stale contents of the shared array, including a
batch that fills the array to its last row followed by a small one; an empty
batch writes 0 like the allocating entry; a batch larger than the array is
refused.

The file name sorts last so that a run stopping at the first failure has run
every other test already; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144


def dev_alloc(rt, nbytes):
    p = ctypes.c_void_p()
    assert rt.lib.tp_alloc(int(nbytes), ctypes.byref(p)) == 0
    return p.value


def upload(rt, arr):
    arr = np.ascontiguousarray(arr, np.float32)
    p = dev_alloc(rt, arr.nbytes)
    assert rt.lib.tp_memcpy_h2d(ctypes.c_void_p(p), arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes) == 0
    return p


def read_one(rt, p):
    out = np.zeros(1, np.float32)
    assert rt.lib.tp_memcpy_d2h(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(p), 4) == 0
    return float(out[0])


def test_noalloc_mean_matches_allocating_entry_twice(cuda_rt):
    rt = cuda_rt
    rng = np.random.default_rng(2024)
    out_ref, out_new = dev_alloc(rt, 4), dev_alloc(rt, 4)
    # calls in a row with different shapes and values; the array's full size
    # (every row slot used) comes before a smaller call, which must not see
    # anything the larger one left behind
    for B, C in ((1024, 10), (37, 1000), (MAX_ROWS, 4), (5, 3)):
        logits = upload(rt, rng.standard_normal((B, C)) * 3)
        targets = upload(rt, rng.integers(0, C, B).astype(np.float32))
        rows = dev_alloc(rt, B * 4)
        assert rt.lib.tpk_cross_entropy_mean(ctypes.c_void_p(logits), ctypes.c_void_p(targets),
                                             ctypes.c_void_p(rows), ctypes.c_void_p(out_ref), B, C) == 0
        assert rt.lib.tpk_cross_entropy_mean_noalloc(ctypes.c_void_p(logits), ctypes.c_void_p(targets),
                                                     ctypes.c_void_p(out_new), B, C) == 0
        want, got = read_one(rt, out_ref), read_one(rt, out_new)
        assert got == pytest.approx(want, rel=1e-5), (B, C, got, want)
        for p in (logits, targets, rows):
            rt.lib.tp_free(ctypes.c_void_p(p))
    rt.lib.tp_free(ctypes.c_void_p(out_ref))
    rt.lib.tp_free(ctypes.c_void_p(out_new))


def test_noalloc_empty_batch_writes_zero_like_allocating_entry(cuda_rt):
    rt = cuda_rt
    out_ref, out_new = dev_alloc(rt, 4), dev_alloc(rt, 4)
    ones = upload(rt, np.ones(1, np.float32))
    for p in (out_ref, out_new):  # a nonzero value first, so a write of 0 shows
        assert rt.lib.tp_memcpy_d2d(ctypes.c_void_p(p), ctypes.c_void_p(ones), 4) == 0
    rows = dev_alloc(rt, 4)
    assert rt.lib.tpk_cross_entropy_mean(ctypes.c_void_p(ones), ctypes.c_void_p(ones), ctypes.c_void_p(rows),
                                         ctypes.c_void_p(out_ref), 0, 10) == 0
    assert rt.lib.tpk_cross_entropy_mean_noalloc(ctypes.c_void_p(ones), ctypes.c_void_p(ones),
                                                 ctypes.c_void_p(out_new), 0, 10) == 0
    assert read_one(rt, out_ref) == 0.0 and read_one(rt, out_new) == 0.0
    for p in (out_ref, out_new, ones, rows):
        rt.lib.tp_free(ctypes.c_void_p(p))


def test_noalloc_refuses_batches_beyond_its_array(cuda_rt):
    rt = cuda_rt
    status = rt.lib.tpk_cross_entropy_mean_noalloc(None, None, None, MAX_ROWS + 1, 10)
    assert status != 0
    assert b"outside" in rt.lib.tp_last_error()
