"""The VGG-11-BN training step (tpcuda.vgg) against the same step composed from
the CPU oracle's op restatements: conv2d, BN training forward/backward, ReLU,
max-pool with indices, linear, cross-entropy and the fused SGD step.

Checks the loss, every parameter after the update and the BN running stats,
at 1e-4 relative to each tensor's scale (the bar for conv / norm / matmul).
"""
import math

import numpy as np
import pytest

from vgg_oracle import oracle_backward, oracle_step

pytestmark = pytest.mark.gpu


def close(a, b, rel=1e-4):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(1e-12, float(np.max(np.abs(b))))
    return float(np.max(np.abs(a - b))) <= rel * scale


def device_forward_state(m):
    """Per-block forward tensors of the last device step as NCHW arrays (for
    teacher forcing), whatever layout the step keeps them in."""
    out = []
    for b in m.blocks:
        C, H, W = b["cout"], b["H"], b["W"]
        sv = {"z": m.activation(b["z"], C, H, W).ravel(), "a": m.activation(b["a"], C, H, W).ravel(),
              "mean": m.read(b["mean"], C), "invstd": m.read(b["invstd"], C)}
        if b["pool"]:
            sv["idx"] = m.activation(b["idx"], C, H // 2, W // 2, np.int32).ravel()
            sv["p"] = m.activation(b["p"], C, H // 2, W // 2).ravel()
        sv["out"] = sv["p"] if b["pool"] else sv["a"]
        out.append(sv)
    return out


@pytest.mark.parametrize("batch", [4, 16])
@pytest.mark.parametrize("layout", ["nhwc", "nchw"])
def test_vgg_step_matches_oracle_composition(cuda_rt, oracle_rt, batch, layout):
    """Forward (activations, loss, running stats) against the oracle's own
    forward; backward against the oracle backward driven by the device's
    forward state; then the SGD update (bit-exact given the gradients)."""
    from tpcuda.vgg import VGG11BN
    m = VGG11BN(cuda_rt, batch, seed=3, layout=layout, keep_acts=True)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((batch, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, batch).astype(np.float32)
    m._h2d(m.x, x)
    m._h2d(m.y, y)
    params = {n: (m.param_array(n), s) for n, s, _ in m.param_specs}
    stats = [(m.read(b["rm"], b["cout"]), m.read(b["rv"], b["cout"])) for b in m.blocks]
    loss_o, new_o, stats_o = oracle_step(oracle_rt, m, params, x, y, stats, m.lr, m.momentum, m.wd)
    m.step_eager()
    # forward: loss and BN running statistics
    loss_c = m.read_loss()
    assert math.isclose(loss_c, loss_o, rel_tol=1e-5), (loss_c, loss_o)
    for li, b in enumerate(m.blocks):
        assert close(m.read(b["rm"], b["cout"]), stats_o[li][0], 1e-4)
        assert close(m.read(b["rv"], b["cout"]), stats_o[li][1], 1e-4)
    # backward, teacher-forced: every gradient within 1e-4 of its tensor's scale
    saved = device_forward_state(m)
    logits = m.read(m.logits, batch * 10)
    grads_o = oracle_backward(oracle_rt, m, params, x, y, saved, logits)
    for n in params:
        g_c = m.grad_array(n)
        if n.startswith("conv") and n.endswith(".b"):
            # a conv bias feeding a BN has a gradient that is zero up to rounding
            assert float(np.max(np.abs(g_c - grads_o[n]))) <= 1e-6 * max(1.0, float(np.max(np.abs(g_c)))), n
        else:
            assert close(g_c, grads_o[n], 1e-4), (n, float(np.max(np.abs(g_c - grads_o[n]))),
                                                  float(np.max(np.abs(grads_o[n]))))
    # update: param - lr * (grad + wd * param) with the momentum buffer starting at 0
    for n in params:
        g_c = m.grad_array(n)
        p0 = params[n][0]
        want = p0 - np.float32(m.lr) * (g_c + np.float32(m.wd) * p0)
        assert close(m.param_array(n), want, 1e-6), n
    if layout == "nhwc":
        # the first conv's padded input channels keep exactly zero filters
        o, k = m.offsets["conv0.w"]
        stored = m.read(m.params + 4 * o, k).reshape(64, m.cin0, 3, 3)
        assert not np.any(stored[:, 3:])
    m.close()


def test_vgg_graph_replay_matches_eager(cuda_rt):
    from tpcuda.vgg import VGG11BN
    rng = np.random.default_rng(9)
    x = rng.standard_normal((8, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, 8).astype(np.float32)
    a, b = VGG11BN(cuda_rt, 8, seed=5), VGG11BN(cuda_rt, 8, seed=5)
    for mdl in (a, b):
        mdl._h2d(mdl.x, x)
        mdl._h2d(mdl.y, y)
    for _ in range(3):
        a.step_eager()
    b.capture()  # runs one eager step, then records (does not run) the step
    b.step()     # steps two and three replay the graph
    b.step()
    cuda_rt.synchronize()
    assert a.read_loss() == b.read_loss()
    for n, _, _ in a.param_specs:
        assert np.array_equal(a.param_array(n), b.param_array(n)), n
    a.close()
    b.close()


def test_vgg_loss_decreases(cuda_rt):
    from tpcuda.vgg import VGG11BN
    rng = np.random.default_rng(11)
    m = VGG11BN(cuda_rt, 32, seed=1, lr=0.02)
    m._h2d(m.x, rng.standard_normal((32, 3, 32, 32)).astype(np.float32))
    m._h2d(m.y, rng.integers(0, 10, 32).astype(np.float32))
    losses = []
    for _ in range(8):
        m.step_eager()
        losses.append(m.read_loss())
    assert losses[-1] < losses[0] * 0.7, losses
    m.close()


def test_vgg_fused_pool_step_matches_kept_activations(cuda_rt):
    """The channels-last step that writes only pooled activations (BN, ReLU and
    pool in one pass; the pool backward read in place) gives bit-identical
    losses and parameters to the same step that also stores every full-size
    BN+ReLU activation (the state the oracle comparison reads)."""
    from tpcuda.vgg import VGG11BN
    rng = np.random.default_rng(11)
    x = rng.standard_normal((8, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, 8).astype(np.float32)
    res = []
    for keep in (False, True):
        m = VGG11BN(cuda_rt, 8, seed=5, layout="nhwc", keep_acts=keep)
        assert all(bool(b["a"]) == (keep or not b["pool"]) for b in m.blocks)
        m._h2d(m.x, x)
        m._h2d(m.y, y)
        losses = []
        for _ in range(2):
            m.step_eager()
            losses.append(m.read_loss())
        res.append((losses, {n: m.param_array(n) for n, _, _ in m.param_specs}))
        m.close()
    assert res[0][0] == res[1][0]
    for n in res[0][1]:
        assert np.array_equal(res[0][1][n], res[1][1][n]), n


@pytest.mark.parametrize("batch", [8, 128])
def test_vgg_step_same_with_and_without_dependent_launch(cuda_rt, batch):
    """Programmatic dependent launch only changes when CTAs are scheduled: the
    graph-replayed step captured with it gives the same bits as the step
    captured in plain stream order."""
    from tpcuda._lib import check
    from tpcuda.vgg import VGG11BN
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, batch).astype(np.float32)
    res = []
    try:
        for pdl in (1, 0):
            check(cuda_rt.lib.tp_set_pdl(pdl))
            m = VGG11BN(cuda_rt, batch, seed=4)
            m._h2d(m.x, x)
            m._h2d(m.y, y)
            m.capture()
            losses = []
            for _ in range(3):
                m.step()
                losses.append(m.read_loss())
            cuda_rt.synchronize()
            res.append((losses, {n: m.param_array(n) for n, _, _ in m.param_specs}))
            m.close()
    finally:
        check(cuda_rt.lib.tp_set_pdl(1))
    assert res[0][0] == res[1][0]
    for n in res[0][1]:
        assert np.array_equal(res[0][1][n], res[1][1][n]), n


@pytest.mark.parametrize("batch", [8, 128])
def test_vgg_per_bucket_update_same_as_one_update(cuda_rt, batch):
    """Updating each gradient bucket on the side stream as soon as its gradients
    are final (the data-parallel schedule, forced here on one GPU) gives the
    same bits as one SGD launch over every parameter at the end of the step:
    the side stream's waits order every update after its gradients' writers
    and its filters' last reader."""
    from tpcuda.vgg import VGG11BN
    rng = np.random.default_rng(batch + 1)
    x = rng.standard_normal((batch, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, batch).astype(np.float32)
    res = []
    for early in (True, False):
        m = VGG11BN(cuda_rt, batch, seed=5, early_update=early, bucket_bytes=1 << 20)
        assert bool(m.bucket_groups) == early
        m._h2d(m.x, x)
        m._h2d(m.y, y)
        losses = []
        m.step_eager()
        losses.append(m.read_loss())
        m.capture()
        for _ in range(3):
            m.step()
            losses.append(m.read_loss())
        cuda_rt.synchronize()
        res.append((losses, {n: m.param_array(n) for n, _, _ in m.param_specs}))
        m.close()
    assert res[0][0] == res[1][0]
    for n in res[0][1]:
        assert np.array_equal(res[0][1][n], res[1][1][n]), n
