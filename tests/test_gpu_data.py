"""Input pipeline on the device: pinned uploads on the copy stream, deferred
stream waits, and the row gather behind the patched DataLoader, bit-exact
against numpy."""
import numpy as np
import pytest

from tpcuda.data import PinnedLoader

pytestmark = pytest.mark.gpu


def test_pinned_loader_delivers_exact_batches_while_kernels_run(cuda_rt):
    rt = cuda_rt
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1000, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, 1000).astype(np.int64)
    ld = PinnedLoader(rt, [x, y], batch_size=96, shuffle=True, dtypes=["float32", "int64"], seed=11, depth=2)
    order = np.random.default_rng(11).permutation(1000)
    for k, (hx, hy) in enumerate(ld):
        idx = order[k * 96:(k + 1) * 96]
        # a kernel that reads the batch right away: it must see the copied values
        s = rt.sumDim(rt.reshape(hx["id"], [len(idx), 3 * 32 * 32])["id"], 1, False)
        got = rt.toNumpy(s["id"])
        np.testing.assert_allclose(got, x[idx].reshape(len(idx), -1).sum(1), rtol=1e-5, atol=1e-4)
        assert np.array_equal(rt.toNumpy(hx["id"]).reshape(x[idx].shape), x[idx])
        assert np.array_equal(rt.toNumpy(hy["id"]), y[idx].astype(np.float32))
        assert hy["dtype"] == "int64"
        for h in (hx, hy, s):
            rt.destroy(h["id"])
    ld.close()


def test_upload_requires_pinned_memory(cuda_rt):
    a = np.zeros(16, np.float32)
    with pytest.raises(RuntimeError, match="pinned"):
        cuda_rt.tensorFromHostAsync(a.ctypes.data, [16])


@pytest.mark.parametrize("shape", [[37, 5], [64, 3, 8, 8], [10]])
def test_gather_rows(cuda_rt, shape):
    rng = np.random.default_rng(len(shape))
    x = rng.standard_normal(shape).astype(np.float32)
    h = cuda_rt.tensorFromData(x.ravel(), shape, "float32")
    rows = rng.integers(0, shape[0], 23)
    g = cuda_rt.gatherRows(h["id"], rows)
    assert g["shape"] == [23] + shape[1:]
    assert np.array_equal(cuda_rt.toNumpy(g["id"]).reshape(g["shape"]), x[rows])
    with pytest.raises(RuntimeError, match="out of bounds"):
        cuda_rt.gatherRows(h["id"], [shape[0]])


def test_bytes_roundtrip(cuda_rt):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((33, 7)).astype(np.float32)
    h = cuda_rt.tensorFromData(x.ravel(), [33, 7], "float32")
    raw = cuda_rt.toBytes(h["id"])
    assert raw == x.astype("<f4").tobytes()
    back = cuda_rt.fromBytes(raw, [33, 7], "float32")
    assert np.array_equal(cuda_rt.toNumpy(back["id"]), x.ravel())
    ints = np.array([3, -2, 0, 7, 2 ** 20], np.int64)
    hi = cuda_rt.fromBytes(ints.astype("<i8").tobytes(), [5], "int64", "int64")
    assert cuda_rt.toBytes(hi["id"], "int64") == ints.astype("<i8").tobytes()
