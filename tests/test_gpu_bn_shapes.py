"""BatchNorm training on NCHW tensors (statistics, finish, normalise; then the
backward sums, finish, apply) against the CPU oracle on shapes that take
every branch: planes whose size is not a multiple of 4 (5x5, 1x1: one value
per step) and those that are (16-byte vectors), channel counts that do not
fill the GPU, images that do not divide evenly between the statistics CTAs,
the fused ReLU forward and the ReLU-masked backward (relu_src).

Tolerance: 1e-4 of the output's scale for y / dx / dgamma / dbeta, 1e-5 for
the statistics and running statistics (the f64 sums make them near exact).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [[8, 16, 5, 5], [6, 4, 1, 1], [4, 64, 32, 32], [33, 24, 12, 12], [7, 3, 4, 4], [64, 40, 28, 28],
          [2, 5, 64, 64]]


def _dev(rt, a):
    a = np.ascontiguousarray(a, np.float32)
    return rt.tensorFromData(a.ravel(), list(a.shape), "float32")


def _orc(orc, a):
    a = np.ascontiguousarray(a, np.float32)
    return orc.tensorFromData(a.ravel().tolist(), list(a.shape), "float32")


def _close(got, want, rel, what):
    scale = max(1e-30, float(np.max(np.abs(want))))
    err = float(np.max(np.abs(got.astype(np.float64) - want)))
    assert err <= rel * scale, (what, err, scale)


def _run_cuda(rt, x, w, b, gy, relu):
    C = x.shape[1]
    hx, hw, hb, hg = _dev(rt, x), _dev(rt, w), _dev(rt, b), _dev(rt, gy)
    rm, rv = _dev(rt, np.zeros(C)), _dev(rt, np.ones(C))
    y, m, s = rt.batchNormTrain(hx["id"], hw["id"], hb["id"], rm["id"], rv["id"], 1e-5, 0.1, relu)
    d = rt.batchNormBackward(hg["id"], hx["id"], hw["id"], m["id"], s["id"], y["id"] if relu else None)
    out = {k: rt.toNumpy(h["id"]).reshape(h["shape"]) for k, h in
           (("y", y), ("mean", m), ("invstd", s), ("rm", rm), ("rv", rv), ("dx", d[0]), ("dw", d[1]), ("db", d[2]))}
    for h in (hx, hw, hb, hg, rm, rv, y, m, s, *d):
        rt.destroy(h["id"])
    return out


def _run_oracle(orc, x, w, b, gy, relu):
    C = x.shape[1]
    ox, ow, ob = _orc(orc, x), _orc(orc, w), _orc(orc, b)
    rm, rv = _orc(orc, np.zeros(C)), _orc(orc, np.ones(C))
    y, m, s = orc.batchNormTrain(ox["id"], ow["id"], ob["id"], rm["id"], rv["id"], 1e-5, 0.1)
    yv = orc.array(y["id"]).reshape(x.shape)
    if relu:
        gy = np.where(yv > 0, gy, 0.0)   # the ReLU backward folded into the BN backward
        yv = np.maximum(yv, 0.0)
    og = _orc(orc, gy)
    d = orc.batchNormBackward(og["id"], ox["id"], ow["id"], m["id"], s["id"])
    out = {"y": yv, "mean": orc.array(m["id"]), "invstd": orc.array(s["id"]), "rm": orc.array(rm["id"]),
           "rv": orc.array(rv["id"]), "dx": orc.array(d[0]["id"]), "dw": orc.array(d[1]["id"]),
           "db": orc.array(d[2]["id"])}
    for h in (ox, ow, ob, rm, rv, y, m, s, og, *d):
        orc.destroy(h["id"])
    return out


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("relu", [False, True])
def test_bn_train_matches_oracle(cuda_rt, oracle_rt, shape, relu):
    rng = np.random.default_rng(sum(shape) + relu)
    C = shape[1]
    x = (rng.standard_normal(shape) * 1.5 + 0.7).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    gy = rng.standard_normal(shape).astype(np.float32)
    want = _run_oracle(oracle_rt, x, w, b, gy, relu)
    got = _run_cuda(cuda_rt, x, w, b, gy, relu)
    for k in ("y", "dx", "dw", "db"):
        _close(got[k].ravel(), want[k].ravel(), 1e-4, k)
    for k in ("mean", "invstd", "rm", "rv"):
        _close(got[k].ravel(), want[k].ravel(), 1e-5, k)


# The one-launch form (statistics and normalisation as work items claimed in a
# fixed order, tp_set_bn_flow) runs by default only on tensors of 32 MB or
# more; mode 2 forces it on these shapes.  Lags of 1 and 3 channels make
# apply items wait for their channel's sums (and more channels than the lag),
# 1 and 4 CTAs per SM change which CTA takes which item.  An item covers about
# 16 K values of one channel: [64, 40, 28, 28] (20 + 20 + 20 + 4 images) and
# [37, 9, 32, 32] (16 + 16 + 5) end in a short range, [512, 6, 8, 8] has two
# full ranges, the others one range per channel.
FLOW_SHAPES = [s for s in SHAPES if (s[2] * s[3]) % 4 == 0] + [[37, 9, 32, 32], [512, 6, 8, 8]]


@pytest.mark.parametrize("shape", FLOW_SHAPES)
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("lag,ctas", [(0, 0), (1, 4), (3, 1)])
def test_bn_one_launch_matches_oracle(cuda_rt, oracle_rt, shape, relu, lag, ctas):
    import ctypes
    rng = np.random.default_rng(sum(shape) + 2 * relu + 7 * lag)
    C = shape[1]
    x = (rng.standard_normal(shape) * 1.5 + 0.7).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    gy = rng.standard_normal(shape).astype(np.float32)
    want = _run_oracle(oracle_rt, x, w, b, gy, relu)
    lib = cuda_rt.lib
    assert lib.tp_set_bn_flow(2, lag, ctas, 0) == 0
    try:
        got = _run_cuda(cuda_rt, x, w, b, gy, relu)
    finally:
        assert lib.tp_set_bn_flow(1, 0, 0, 0) == 0
    status = ctypes.c_int(-1)
    assert lib.tp_gemm_status(ctypes.byref(status), 1) == 0 and status.value == 0, "a bounded wait expired"
    for k in ("y", "dx", "dw", "db"):
        _close(got[k].ravel(), want[k].ravel(), 1e-4, k)
    for k in ("mean", "invstd", "rm", "rv"):
        _close(got[k].ravel(), want[k].ravel(), 1e-5, k)


def test_bn_flow_switch_rejects_bad_values(cuda_rt):
    lib = cuda_rt.lib
    assert lib.tp_set_bn_flow(3, 0, 0, 0) != 0
    assert lib.tp_set_bn_flow(1, -1, 0, 0) != 0
    assert lib.tp_set_bn_flow(1, 0, 9, 0) != 0
    assert lib.tp_set_bn_flow(1, 0, 0, 0) == 0
