"""Sanity checks of the oracle's restatements against numpy (CPU only)."""
import numpy as np
import pytest

import oracle_runtime as O


def test_matmul_matches_numpy():
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (17, 33)).astype(np.float32)
    B = rng.uniform(-1, 1, (33, 9)).astype(np.float32)
    C = O.matmul2d(A.ravel(), B.ravel(), 17, 33, 9).reshape(17, 9)
    np.testing.assert_allclose(C, A.astype(np.float64) @ B.astype(np.float64), rtol=1e-5, atol=1e-5)


def test_softmax_and_logsoftmax_match_numpy(oracle_rt):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 7)).astype(np.float32)
    h = oracle_rt.tensorFromData(x.ravel().tolist(), [5, 7], "float32")
    s = np.asarray(oracle_rt.toList(oracle_rt.softmax(h["id"], -1)["id"])).reshape(5, 7)
    ls = np.asarray(oracle_rt.toList(oracle_rt.logSoftmax(h["id"], -1)["id"])).reshape(5, 7)
    e = np.exp(x - x.max(1, keepdims=True))
    ref = e / e.sum(1, keepdims=True)
    np.testing.assert_allclose(s, ref, rtol=1e-5)
    np.testing.assert_allclose(ls, np.log(ref), rtol=1e-5, atol=1e-6)


def test_conv_backward_consistent_with_forward(oracle_rt):
    """<conv(x), dy> is bilinear: d/dx and d/dw from the backward kernels match
    finite differences of the forward kernel on a tiny case."""
    rng = np.random.default_rng(2)
    x = rng.standard_normal((2, 3, 6, 5)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32)
    p = O.conv_params(x.shape, w.shape, [1], [1])
    out = np.empty(2 * 4 * p.OH * p.OW, np.float32)
    b = np.zeros(4, np.float32)
    import ctypes
    O.lib().or_conv2d(O.fp(x.ravel()), O.fp(w.ravel()), O.fp(b), O.fp(out), ctypes.byref(p))
    dy = rng.standard_normal(out.shape).astype(np.float32)
    dx = np.empty(x.size, np.float32)
    dw = np.empty(w.size, np.float32)
    O.lib().or_conv2d_input_backward(O.fp(dy), O.fp(w.ravel()), O.fp(dx), ctypes.byref(p))
    O.lib().or_conv2d_weight_backward(O.fp(dy), O.fp(x.ravel()), O.fp(dw), ctypes.byref(p))
    # bilinearity: <conv(x,w), dy> == <x, dx> == <w, dw>
    s0 = float(np.dot(out.astype(np.float64), dy))
    assert abs(s0 - float(np.dot(x.ravel().astype(np.float64), dx))) < 1e-3 * max(1, abs(s0))
    assert abs(s0 - float(np.dot(w.ravel().astype(np.float64), dw))) < 1e-3 * max(1, abs(s0))


def test_reduce_all_tree_order():
    x = np.arange(1000, dtype=np.float32)
    assert O.lib().or_reduce_all(O.fp(x), x.size, 0) == np.float32(499500.0)
    assert O.lib().or_reduce_all(O.fp(x), x.size, 2) == np.float32(999.0)
    assert abs(O.lib().or_reduce_all(O.fp(x), x.size, 1) - 499.5) < 1e-4


def test_sgd_momentum_buffer_starts_at_zero(oracle_rt):
    """optim/__init__.py:177-179: the buffer starts at zeros, so step 1 gives
    buf = (1-dampening) * g, not g."""
    p = oracle_rt.tensorFromData([1.0, 2.0], [2], "float32")
    g = oracle_rt.tensorFromData([0.5, -0.5], [2], "float32")
    b = oracle_rt.zeros([2], "float32")
    oracle_rt.sgdStep(p["id"], g["id"], b["id"], 0.1, 0.9, 0.0, 0.5, False)
    assert oracle_rt.toList(b["id"]) == pytest.approx([0.25, -0.25])
    assert oracle_rt.toList(p["id"]) == pytest.approx([1.0 - 0.025, 2.0 + 0.025])
