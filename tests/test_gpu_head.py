"""The one-launch classifier head (tpk_linear_cross_entropy_step): linear
layer, mean cross-entropy and their gradients.

* The cross-entropy arithmetic on the kernel's own logits against the
  oracle's restatement of cross_entropy.wgsl / cross_entropy_backward.wgsl
  (per-row losses and dlogits to 1e-6 of scale, targets outside [0, K)
  clamped as the shader does).
* The contractions (logits, dx = g w, dw = g^T x, db = sum g) against float64
  numpy on the same inputs, 1e-5 of scale.
* The per-op composition the VGG step used before (tpk_gemm, tpk_cross_entropy_mean,
  tpk_cross_entropy_backward, tpk_gemm x 2, tpk_channel_sum): same values to 1e-5.
* Repeated calls are bit-identical (fixed-order sums), the ticket survives
  grids of 1 and 16 CTAs back to back, NULL outputs are skipped, and the
  limits are checked.
"""
import ctypes

import numpy as np
import pytest

from tpcuda._lib import check

pytestmark = pytest.mark.gpu


def _p(rt, h):
    return ctypes.c_void_p(rt.devicePtr(h["id"])) if h is not None else None


def _dev(rt, a):
    a = np.ascontiguousarray(a, np.float32)
    return rt.tensorFromData(a.ravel(), list(a.shape), "float32")


def _run(rt, x, w, b, t, outputs=("logits", "rows", "mean", "dx", "dw", "db")):
    B, F = x.shape
    K = w.shape[0]
    hx, hw, ht = _dev(rt, x), _dev(rt, w), _dev(rt, t)
    hb = _dev(rt, b) if b is not None else None
    shapes = {"logits": [B, K], "rows": [B], "mean": [1], "dx": [B, F], "dw": [K, F], "db": [K]}
    outs = {k: (rt.full(shapes[k], -7.0, "float32") if k in outputs else None) for k in shapes}
    check(rt.lib.tpk_linear_cross_entropy_step(_p(rt, hx), _p(rt, hw), _p(rt, hb), _p(rt, ht),
                                               *[_p(rt, outs[k]) for k in ("logits", "rows", "mean", "dx", "dw", "db")],
                                               B, F, K, 1.0 / B))
    res = {k: rt.toNumpy(h["id"]).reshape(shapes[k]) for k, h in outs.items() if h is not None}
    for h in [hx, hw, ht, hb] + list(outs.values()):
        if h is not None:
            rt.destroy(h["id"])
    return res


def _close(got, want, rel, what):
    scale = max(1e-30, float(np.max(np.abs(want))))
    err = float(np.max(np.abs(np.asarray(got, np.float64) - want)))
    assert err <= rel * scale, (what, err, scale)


def _inputs(B, F, K, seed, bias=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, F)).astype(np.float32)
    w = (rng.standard_normal((K, F)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(K) * 0.1).astype(np.float32) if bias else None
    t = rng.integers(0, K, B).astype(np.float32)
    t[: min(B, 3)] = [-1.0, K + 2.0, K - 1.0][: min(B, 3)]  # clamped to 0 and K-1
    return x, w, b, t


@pytest.mark.parametrize("B,F,K", [(1024, 512, 10), (128, 512, 10), (1000, 100, 7), (7, 1024, 32), (1, 33, 1),
                                   (300, 256, 10), (1025, 512, 10), (20000, 64, 17)])
def test_head_matches_oracle_and_float64(cuda_rt, oracle_rt, B, F, K):
    x, w, b, t = _inputs(B, F, K, B + F + K)
    r = _run(cuda_rt, x, w, b, t)
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    logits = x64 @ w64.T + b
    _close(r["logits"], logits, 1e-5, "logits")
    # cross-entropy on the kernel's own logits: the oracle's restatement of the shaders
    orc = oracle_rt
    ol = orc.tensorFromData(r["logits"].ravel().tolist(), [B, K], "float32")
    ot = orc.tensorFromData(t.tolist(), [B], "float32")
    rows = orc.array(orc.crossEntropy(ol["id"], ot["id"])["id"])
    one = orc.tensorFromData([1.0], [1], "float32")
    g = orc.array(orc.crossEntropyBackward(one["id"], ol["id"], ot["id"], "mean")["id"]).reshape(B, K)
    _close(r["rows"], rows.astype(np.float64), 1e-6, "loss rows")
    _close(r["mean"], np.array([rows.astype(np.float64).mean()]), 1e-6, "loss mean")
    g64 = g.astype(np.float64)
    _close(r["dx"], g64 @ w64, 1e-5, "dx")
    _close(r["dw"], g64.T @ x64, 1e-5, "dw")
    _close(r["db"], g64.sum(0), 1e-5, "db")


def test_head_matches_per_op_composition(cuda_rt):
    rt = cuda_rt
    B, F, K = 1024, 512, 10
    x, w, b, t = _inputs(B, F, K, 5)
    r = _run(rt, x, w, b, t)
    hx, hw, hb, ht = _dev(rt, x), _dev(rt, w), _dev(rt, b), _dev(rt, t)
    lo, rows, mean = rt.zeros([B, K], "float32"), rt.zeros([B], "float32"), rt.zeros([1], "float32")
    g, dx, dw, db = (rt.zeros(s, "float32") for s in ([B, K], [B, F], [K, F], [K]))
    L, P = rt.lib, lambda h: _p(rt, h)  # noqa: E731
    check(L.tpk_gemm(P(hx), 0, P(hw), 1, P(lo), B, K, F, P(hb)))
    check(L.tpk_cross_entropy_mean(P(lo), P(ht), P(rows), P(mean), B, K))
    check(L.tpk_cross_entropy_backward(P(lo), P(ht), P(g), B, K, 1.0 / B))
    check(L.tpk_gemm(P(g), 1, P(hx), 0, P(dw), K, F, B, None))
    check(L.tpk_channel_sum(P(g), B, K, 1, P(db)))
    check(L.tpk_gemm(P(g), 0, P(hw), 0, P(dx), B, F, K, None))
    for k, h in (("logits", lo), ("rows", rows), ("mean", mean), ("dx", dx), ("dw", dw), ("db", db)):
        _close(r[k], rt.toNumpy(h["id"]).reshape(r[k].shape).astype(np.float64), 1e-5, k)


def test_head_is_deterministic_and_skips_null_outputs(cuda_rt):
    x, w, b, t = _inputs(1024, 512, 10, 9)
    a = _run(cuda_rt, x, w, b, t)
    small = _inputs(5, 512, 10, 10)  # one CTA: the tickets wrap at different counts
    _run(cuda_rt, *small)
    ragged = _inputs(1000, 512, 10, 11)  # 125 CTAs: a last group of 5
    _run(cuda_rt, *ragged)
    c = _run(cuda_rt, x, w, b, t)
    for k in a:
        assert np.array_equal(a[k], c[k]), k
    only = _run(cuda_rt, x, w, None, t, outputs=("mean", "dw"))
    assert set(only) == {"mean", "dw"}
    nb = _run(cuda_rt, x, w, None, t)
    assert np.array_equal(only["mean"], nb["mean"]) and np.array_equal(only["dw"], nb["dw"])


def test_head_limits(cuda_rt):
    x, w, b, t = _inputs(4, 16, 33, 1)
    with pytest.raises(RuntimeError, match="classes"):
        _run(cuda_rt, x, w, b, t)
    x, w, b, t = _inputs(4, 1025, 4, 1)
    with pytest.raises(RuntimeError, match="features"):
        _run(cuda_rt, x, w, b, t)
