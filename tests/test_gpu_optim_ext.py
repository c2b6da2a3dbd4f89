"""The fused RMSprop / Adagrad / Adamax / NAdam / RAdam steps against the
oracle's restatements of rmsprop_step.wgsl and extended_step.wgsl: bit-exact,
per-tensor and multi-tensor, over several steps, with and without weight decay
and momentum, on sizes that leave 16-byte tails and span several chunks."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 5, 4097, 70001, 131072]


def _pair(cu, orc, a):
    a = np.ascontiguousarray(a, np.float32)
    return cu.tensorFromData(a.ravel(), list(a.shape), "float32"), orc.tensorFromData(a.ravel(), list(a.shape),
                                                                                      "float32")


def _hp(kind, step, wd):
    b1, b2 = 0.9, 0.999
    if kind == "rmsprop":
        return (0.01, 0.99, 1e-8, wd, 0.9 if step % 2 else 0.0)
    if kind == "rmsprop_m":
        return (0.01, 0.99, 1e-8, wd, 0.9)
    if kind == "adagrad":
        return (0.01 / (1.0 + (step - 1) * 0.01), 1e-10, wd)
    bc1 = 1.0 - b1 ** step
    if kind == "adamax":
        return (0.002, b1, b2, 1e-8, wd, 0.002 / bc1, 1.0)
    if kind == "nadam":
        mu_next = b1 * (1.0 - 0.5 * (0.96 ** ((step + 1) * 4e-3)))
        return (0.002, b1, b2, 1e-8, wd, 0.002 / bc1, mu_next)
    return (1e-3, b1, b2, 1e-8, wd, 1e-3 / bc1, b1 ** step, b2 ** step, step)


METHOD = {"rmsprop": "rmspropStep", "rmsprop_m": "rmspropStep", "adagrad": "adagradStep", "adamax": "adamaxStep",
          "nadam": "nadamStep", "radam": "radamStep"}
NSTATE = {"adagrad": 1}


@pytest.mark.parametrize("kind", ["rmsprop", "rmsprop_m", "adagrad", "adamax", "nadam", "radam"])
@pytest.mark.parametrize("multi", [False, True])
@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_fused_step_bit_exact(cuda_rt, oracle_rt, kind, multi, wd):
    cu, orc = cuda_rt, oracle_rt
    rng = np.random.default_rng(len(kind) * 7 + int(multi) + int(wd * 100))
    ns = NSTATE.get(kind, 2)
    tensors = []
    for n in SIZES:
        p = _pair(cu, orc, rng.standard_normal(n) * 0.1)
        states = [_pair(cu, orc, np.zeros(n) if k == 0 else np.zeros(n)) for k in range(ns)]
        tensors.append((n, p, states))
    # RAdam's rectified branch (rho_t > 5) starts at step 6 with beta2 = 0.999
    steps = 8 if kind == "radam" else 4
    for step in range(1, steps + 1):
        grads = [_pair(cu, orc, rng.standard_normal(n) * 1e-2) for n, _, _ in tensors]
        hp = _hp(kind, step, wd)
        name = METHOD[kind]
        for side, rt in ((0, cu), (1, orc)):
            ps = [t[1][side]["id"] for t in tensors]
            gs = [g[side]["id"] for g in grads]
            sts = [[t[2][k][side]["id"] for t in tensors] for k in range(ns)]
            if multi:
                getattr(rt, name + "Multi")(ps, gs, *sts, *hp)
            else:
                for i in range(len(ps)):
                    getattr(rt, name)(ps[i], gs[i], *[s[i] for s in sts], *hp)
    for n, p, states in tensors:
        assert np.array_equal(cu.toNumpy(p[0]["id"]), orc.array(p[1]["id"])), (kind, n, "param")
        for k, st in enumerate(states):
            if kind == "rmsprop" and k == 1:
                continue  # alternates momentum on and off: the buffer is compared in rmsprop_m
            assert np.array_equal(cu.toNumpy(st[0]["id"]), orc.array(st[1]["id"])), (kind, n, "state", k)


def test_length_mismatch_is_an_error(cuda_rt):
    a = cuda_rt.zeros([4], "float32")
    b = cuda_rt.zeros([5], "float32")
    with pytest.raises(RuntimeError, match="lengths must match"):
        cuda_rt.nadamStep(a["id"], b["id"], a["id"], a["id"], 1e-3, 0.9, 0.999, 1e-8, 0.0, 1e-2, 0.9)


def test_radam_uses_the_step_count(cuda_rt):
    """The step count selects the rectified branch: at step 6 (beta2 0.999)
    rho_t > 5, so the update differs from the one with the count dropped to 1."""
    cu = cuda_rt
    outs = []
    for step in (6, 0):
        p = cu.tensorFromData(np.ones(8, np.float32), [8], "float32")
        g = cu.tensorFromData(np.full(8, 0.5, np.float32), [8], "float32")
        m, v = cu.zeros([8], "float32"), cu.zeros([8], "float32")
        cu.radamStep(p["id"], g["id"], m["id"], v["id"], 1e-3, 0.9, 0.999, 1e-8, 0.0, 1e-3 / (1 - 0.9 ** 6),
                     0.9 ** 6, 0.999 ** 6, step)
        outs.append(cu.toNumpy(p["id"]))
    assert not np.array_equal(outs[0], outs[1])
    assert math.isfinite(float(outs[0][0]))
