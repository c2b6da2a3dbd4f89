"""Contractions, pooling and normalisation: CUDA runtime vs the CPU oracle.

Tolerance for matmul / conv / norms / reductions: 1e-4 relative to the output
scale (max |reference| of the tensor), the bar stated for this path; pooling
values and indices are bit-exact.
"""
import numpy as np
import pytest

from test_gpu_ops import both, check, vals

pytestmark = pytest.mark.gpu


def close_scaled(cuda_rt, oracle_rt, hc, ho, rel=1e-4):
    assert hc["shape"] == ho["shape"], (hc, ho)
    a, b = vals(cuda_rt, hc), vals(oracle_rt, ho)
    scale = max(1e-30, float(np.max(np.abs(b)))) if b.size else 1.0
    err = float(np.max(np.abs(a - b))) if b.size else 0.0
    assert err <= rel * scale, (err, scale)


@pytest.mark.parametrize("sa,sb", [([7, 5], [5, 3]), ([64, 784], [784, 10]), ([130, 257], [257, 129]),
                                   ([5], [5, 4]), ([6, 5], [5]), ([3, 17, 9], [3, 9, 11]), ([2, 3, 8], [8, 5]),
                                   ([1, 1], [1, 1]), ([300, 2048], [2048, 70])])
def test_matmul(cuda_rt, oracle_rt, sa, sb):
    rng = np.random.default_rng(sum(sa) + sum(sb))
    ca, oa = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, sa))
    cb, ob = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, sb))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.matmul(ca["id"], cb["id"]), oracle_rt.matmul(oa["id"], ob["id"]))


def test_matmul_shape_error(cuda_rt):
    a = cuda_rt.zeros([2, 3], "float32")
    b = cuda_rt.zeros([4, 5], "float32")
    with pytest.raises(RuntimeError, match="matmul dimension mismatch"):
        cuda_rt.matmul(a["id"], b["id"])


def test_linear_matches_transpose_matmul_add(cuda_rt, oracle_rt):
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (33, 70)).astype(np.float32)
    w = rng.uniform(-1, 1, (19, 70)).astype(np.float32)
    b = rng.uniform(-1, 1, (19,)).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    cw, ow = both(cuda_rt, oracle_rt, w)
    cb, ob = both(cuda_rt, oracle_rt, b)
    y = cuda_rt.linear(cx["id"], cw["id"], cb["id"])
    ref = oracle_rt.add(oracle_rt.matmul(ox["id"], oracle_rt.transpose2d(ow["id"])["id"])["id"], ob["id"])
    close_scaled(cuda_rt, oracle_rt, y, ref)


CONV_CASES = [
    # x shape, w shape, stride, padding, groups
    ([2, 3, 8, 8], [4, 3, 3, 3], [1], [1], 1),
    ([1, 1, 5, 5], [1, 1, 3, 3], [1], [1], 1),
    ([4, 8, 14, 14], [16, 8, 3, 3], [1], [1], 1),
    ([2, 3, 17, 15], [8, 3, 7, 7], [2], [3], 1),
    ([2, 4, 9, 9], [6, 2, 3, 3], [1], [0], 2),
    ([3, 5, 6, 7], [7, 5, 1, 1], [1], [0], 1),
    ([2, 16, 4, 4], [32, 16, 3, 3], [1], [1], 1),
    ([8, 64, 16, 16], [128, 64, 3, 3], [1], [1], 1),
]


@pytest.mark.parametrize("xs,ws,st,pd,g", CONV_CASES)
def test_conv2d_forward(cuda_rt, oracle_rt, xs, ws, st, pd, g):
    rng = np.random.default_rng(sum(xs))
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(xs))
    cw, ow = both(cuda_rt, oracle_rt, rng.standard_normal(ws) * 0.3)
    bias = rng.standard_normal(ws[0]).astype(np.float32).tolist()
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2d(cx["id"], cw["id"], bias, st, pd, [1], g),
                 oracle_rt.conv2d(ox["id"], ow["id"], bias, st, pd, [1], g))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2d(cx["id"], cw["id"], None, st, pd, [1], g),
                 oracle_rt.conv2d(ox["id"], ow["id"], None, st, pd, [1], g))


@pytest.mark.parametrize("xs,ws,st,pd,g", [c for c in CONV_CASES if c[4] == 1])
def test_conv2d_backward(cuda_rt, oracle_rt, xs, ws, st, pd, g):
    rng = np.random.default_rng(sum(ws))
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(xs))
    cw, ow = both(cuda_rt, oracle_rt, rng.standard_normal(ws) * 0.3)
    y = oracle_rt.conv2d(ox["id"], ow["id"], None, st, pd, [1], 1)
    gy = rng.standard_normal(y["shape"])
    cg, og = both(cuda_rt, oracle_rt, gy)
    ys = y["shape"]
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dInputBackward(cg["id"], cw["id"], xs, ys, st, pd),
                 oracle_rt.conv2dInputBackward(og["id"], ow["id"], xs, ys, st, pd))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dWeightBackward(cg["id"], cx["id"], ws, ys, xs, st, pd),
                 oracle_rt.conv2dWeightBackward(og["id"], ox["id"], ws, ys, xs, st, pd))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dBiasBackward(cg["id"], ws[0], ys),
                 oracle_rt.conv2dBiasBackward(og["id"], ws[0], ys))


POOL_CASES = [([2, 3, 8, 8], [2], [2], [0], [1]), ([1, 2, 7, 9], [3], [2], [1], [1]),
              ([2, 2, 6, 6], [3, 2], [1, 1], [1, 0], [1]), ([4, 16, 14, 14], [2], [], [0], [1]),
              ([1, 1, 9, 9], [2], [2], [0], [2]), ([64, 8, 28, 28], [2], [2], [0], [1])]


@pytest.mark.parametrize("xs,k,s,p,d", POOL_CASES)
def test_maxpool_bit_exact_with_indices_and_backward(cuda_rt, oracle_rt, xs, k, s, p, d):
    rng = np.random.default_rng(sum(xs))
    x = np.round(rng.standard_normal(xs) * 3).astype(np.float32)  # ties exercise the first-max rule
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, cuda_rt.maxPool2d(cx["id"], k, s, p, d), oracle_rt.maxPool2d(ox["id"], k, s, p, d))
    cy, ci = cuda_rt.maxPool2dWithIndices(cx["id"], k, s, p, d)
    oy, oi = oracle_rt.maxPool2dWithIndices(ox["id"], k, s, p, d)
    check(cuda_rt, oracle_rt, cy, oy)
    assert np.array_equal(vals(cuda_rt, ci), vals(oracle_rt, oi))
    gy = rng.standard_normal(cy["shape"])
    cg, og = both(cuda_rt, oracle_rt, gy)
    check(cuda_rt, oracle_rt, cuda_rt.maxPool2dBackward(cg["id"], ci["id"], xs, k, s, p, d),
          oracle_rt.maxPool2dBackward(og["id"], oi["id"], xs, k, s, p, d))


@pytest.mark.parametrize("shape", [[4, 3], [8, 16, 5, 5], [2, 64, 32, 32], [3, 7, 11]])
def test_batchnorm_eval(cuda_rt, oracle_rt, shape):
    rng = np.random.default_rng(1)
    C = shape[1]
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(shape))
    prm = [both(cuda_rt, oracle_rt, a) for a in (1 + 0.1 * rng.standard_normal(C), 0.1 * rng.standard_normal(C),
                                                 0.1 * rng.standard_normal(C), rng.uniform(0.5, 2, C))]
    check(cuda_rt, oracle_rt, cuda_rt.batchNorm(cx["id"], *[p[0]["id"] for p in prm], 1e-5),
          oracle_rt.batchNorm(ox["id"], *[p[1]["id"] for p in prm], 1e-5), rtol=1e-6, atol=1e-6)
    check(cuda_rt, oracle_rt, cuda_rt.batchNorm(cx["id"], None, None, None, None, 1e-5),
          oracle_rt.batchNorm(ox["id"], None, None, None, None, 1e-5), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("shape", [[16, 8], [8, 16, 5, 5], [4, 64, 32, 32], [2, 3, 7]])
def test_batchnorm_train_forward_backward(cuda_rt, oracle_rt, shape):
    rng = np.random.default_rng(2)
    C = shape[1]
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    cw, ow = both(cuda_rt, oracle_rt, 1 + 0.1 * rng.standard_normal(C))
    cb, ob = both(cuda_rt, oracle_rt, 0.1 * rng.standard_normal(C))
    crm, orm = both(cuda_rt, oracle_rt, np.zeros(C))
    crv, orv = both(cuda_rt, oracle_rt, np.ones(C))
    cy, cm, cs = cuda_rt.batchNormTrain(cx["id"], cw["id"], cb["id"], crm["id"], crv["id"], 1e-5, 0.1)
    oy, om, os_ = oracle_rt.batchNormTrain(ox["id"], ow["id"], ob["id"], orm["id"], orv["id"], 1e-5, 0.1)
    close_scaled(cuda_rt, oracle_rt, cy, oy)
    for c_, o_ in ((cm, om), (cs, os_), (crm, orm), (crv, orv)):
        close_scaled(cuda_rt, oracle_rt, c_, o_, 1e-5)
    gy = rng.standard_normal(shape)
    cg, og = both(cuda_rt, oracle_rt, gy)
    cd = cuda_rt.batchNormBackward(cg["id"], cx["id"], cw["id"], cm["id"], cs["id"])
    od = oracle_rt.batchNormBackward(og["id"], ox["id"], ow["id"], om["id"], os_["id"])
    for c_, o_ in zip(cd, od):
        close_scaled(cuda_rt, oracle_rt, c_, o_)


def test_batchnorm_fused_relu_matches_composition(cuda_rt):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((4, 6, 5, 5)).astype(np.float32)
    h = cuda_rt.tensorFromData(x.ravel(), list(x.shape), "float32")
    y0 = cuda_rt.batchNormTrain(h["id"], None, None, None, None, 1e-5, 0.1)[0]
    y1 = cuda_rt.batchNormTrain(h["id"], None, None, None, None, 1e-5, 0.1, True)[0]
    assert np.array_equal(np.maximum(vals(cuda_rt, y0), 0), vals(cuda_rt, y1))
    gy = cuda_rt.tensorFromData(rng.standard_normal(x.size).astype(np.float32), list(x.shape), "float32")
    _, m, s = cuda_rt.batchNormTrain(h["id"], None, None, None, None, 1e-5, 0.1)
    mask = cuda_rt.gt(y1["id"], cuda_rt.zeros([1], "float32")["id"])
    masked = cuda_rt.mul(gy["id"], mask["id"])
    a = cuda_rt.batchNormBackward(masked["id"], h["id"], None, m["id"], s["id"])[0]
    b = cuda_rt.batchNormBackward(gy["id"], h["id"], None, m["id"], s["id"], y1["id"])[0]
    assert np.array_equal(vals(cuda_rt, a), vals(cuda_rt, b))


# D % 4 == 0 takes the 16-byte kernels (1 / 2 / 4 / 8 float4 per thread; 2052: a
# partly filled last group); hundreds of rows make the dgamma / dbeta column sum
# run over hundreds of per-CTA partial rows
@pytest.mark.parametrize("rows,D", [(4, 10), (33, 300), (16, 1024), (8, 4096), (3, 9000), (600, 2048),
                                    (5000, 512), (64, 8192), (40, 2052), (700, 1030)])
def test_layernorm_forward_backward(cuda_rt, oracle_rt, rows, D):
    rng = np.random.default_rng(5)
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal((rows, D)))
    cg, og = both(cuda_rt, oracle_rt, 1 + 0.1 * rng.standard_normal(D))
    cb, ob = both(cuda_rt, oracle_rt, 0.1 * rng.standard_normal(D))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.layerNorm(cx["id"], [D], cg["id"], cb["id"], 1e-5),
                 oracle_rt.layerNorm(ox["id"], [D], og["id"], ob["id"], 1e-5))
    cy, cm, cr = cuda_rt.layerNormForward(cx["id"], [D], cg["id"], cb["id"], 1e-5)
    oy, om, orr = oracle_rt.layerNormForward(ox["id"], [D], og["id"], ob["id"], 1e-5)
    close_scaled(cuda_rt, oracle_rt, cy, oy)
    cdy, ody = both(cuda_rt, oracle_rt, rng.standard_normal((rows, D)))
    cd = cuda_rt.layerNormBackward(cdy["id"], cx["id"], [D], cg["id"], cm["id"], cr["id"])
    od = oracle_rt.layerNormBackward(ody["id"], ox["id"], [D], og["id"], om["id"], orr["id"])
    for c_, o_ in zip(cd, od):
        close_scaled(cuda_rt, oracle_rt, c_, o_)

