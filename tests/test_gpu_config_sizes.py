"""Parity at the benchmark configurations' full sizes, through the runtime
surface the reference package calls (CudaRuntime, handle API).

At these sizes the tensor-map extents, split-K counts, grid limits and 32-bit
index products differ from the small parity cases, so every op here runs on
the device at its configured size and is checked against the CPU oracle:

* reductions, norms and the softmax forward: the oracle runs at the full size
  too (its C loops finish in about a second each); the softmax backwards, which
  the reference computes in O(C^2) per row, on a seeded sample of 256 rows;
* the contractions: the oracle computes a seeded sample of the output (rows x
  columns of a matmul or linear layer, whole images of a convolution's forward
  and data gradient, a few output channels of a weight gradient); each
  sampled value is the oracle's own per-element arithmetic on the same inputs,
  so the sample is exact, not an estimate;
* the fused optimizer steps over the whole 64-tensor set (402,718,720
  elements, 3 steps from zero moments with regenerated gradients): the oracle
  steps one tensor of each of the four shapes, which must match bit for bit.

Tolerances: 1e-4 relative to the output's scale (max |oracle|) for
contractions, norms and reductions (the weight gradients, whose sums run over
0.4-1.6 M products, also against the exact float64 sum, see below); bit-exact for max / argmax indices and
the optimizer steps.  Inputs come from the device RNG (seeded) and are read
back for the oracle.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-4


def host(rt, h):
    return rt.toNumpy(h["id"]).reshape(h["shape"])


def orc_t(orc, a):
    a = np.ascontiguousarray(a, np.float32)
    return orc.tensorFromData(a.ravel(), list(a.shape), "float32")


def dev_t(rt, a):
    a = np.ascontiguousarray(a, np.float32)
    return rt.tensorFromData(a.ravel(), list(a.shape), "float32")


def randn(rt, shape, seed):
    rt.setSeed(seed)
    return rt.randn(shape, "float32")


def uniform(rt, shape, seed):
    """~U(-1, 1) from the device RNG."""
    rt.setSeed(seed)
    u = rt.rand(shape, "float32")
    v = rt.mulScalar(u["id"], 2.0)
    w = rt.add(v["id"], rt.full([1], -1.0, "float32")["id"])
    for h in (u, v):
        rt.destroy(h["id"])
    return w


def assert_scaled(got, want, rel=REL, what=""):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    scale = max(1e-30, float(np.max(np.abs(want))))
    err = float(np.max(np.abs(got - want)))
    assert err <= rel * scale, (what, err, scale)


def free(rt, *hs):
    for h in hs:
        rt.destroy(h["id"])


# ---- reductions / norms / softmax (configs: reductions and norms) ------------------------------


def test_layernorm_16384x4096_fwd_bwd(cuda_rt, oracle_rt):
    rt, orc = cuda_rt, oracle_rt
    R, D = 16384, 4096
    rng = np.random.default_rng(11)
    gam, bet = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32), (0.1 * rng.standard_normal(D)).astype(np.float32)
    x, dy = randn(rt, [R, D], 101), randn(rt, [R, D], 102)
    g, b = dev_t(rt, gam), dev_t(rt, bet)
    y, m, r = rt.layerNormForward(x["id"], [D], g["id"], b["id"], 1e-5)
    dx, dg, db = rt.layerNormBackward(dy["id"], x["id"], [D], g["id"], m["id"], r["id"])
    ox, ody, og, ob = orc_t(orc, host(rt, x)), orc_t(orc, host(rt, dy)), orc_t(orc, gam), orc_t(orc, bet)
    oy, om, orr = orc.layerNormForward(ox["id"], [D], og["id"], ob["id"], 1e-5)
    odx, odg, odb = orc.layerNormBackward(ody["id"], ox["id"], [D], og["id"], om["id"], orr["id"])
    for c, o, nm in ((y, oy, "y"), (m, om, "mean"), (r, orr, "rstd"), (dx, odx, "dx"), (dg, odg, "dgamma"),
                     (db, odb, "dbeta")):
        assert_scaled(rt.toNumpy(c["id"]), orc.array(o["id"]), what=nm)
    free(rt, x, dy, g, b, y, m, r, dx, dg, db)
    for h in (ox, ody, og, ob, oy, om, orr, odx, odg, odb):
        orc.destroy(h["id"])


def test_softmax_logsoftmax_32768x8192_fwd_bwd(cuda_rt, oracle_rt):
    rt, orc = cuda_rt, oracle_rt
    R, C = 32768, 8192
    x, gy = randn(rt, [R, C], 201), randn(rt, [R, C], 202)
    ox, ogy = orc_t(orc, host(rt, x)), orc_t(orc, host(rt, gy))
    for fwd, bwd in (("softmax", "softmaxBackward"), ("logSoftmax", "logSoftmaxBackward")):
        s = getattr(rt, fwd)(x["id"], -1)
        os_ = getattr(orc, fwd)(ox["id"], -1)
        assert_scaled(rt.toNumpy(s["id"]), orc.array(os_["id"]), what=fwd)
        # the backward from the device's own forward output, on both sides; the
        # reference shader recomputes each row's dot product per element (O(C^2)
        # per row), so the oracle does a seeded sample of rows (rows are independent)
        rows = np.sort(np.random.default_rng(5).choice(R, 254, replace=False))
        rows = np.unique(np.concatenate([[0, R - 1], rows]))
        S, GY = host(rt, s), host(rt, gy)
        os_dev, ogs = orc_t(orc, S[rows]), orc_t(orc, GY[rows])
        d = getattr(rt, bwd)(gy["id"], s["id"], R, C)
        od = getattr(orc, bwd)(ogs["id"], os_dev["id"], len(rows), C)
        assert_scaled(host(rt, d)[rows], orc.array(od["id"]).reshape(len(rows), C), what=bwd)
        orc.destroy(ogs["id"])
        free(rt, s, d)
        for h in (os_, os_dev, od):
            orc.destroy(h["id"])
    free(rt, x, gy)
    orc.destroy(ox["id"])
    orc.destroy(ogy["id"])


def test_sum_mean_max_8192x8192_both_dims(cuda_rt, oracle_rt):
    rt, orc = cuda_rt, oracle_rt
    x = randn(rt, [8192, 8192], 301)
    ox = orc_t(orc, host(rt, x))
    for d in (0, -1):
        for op in ("sumDim", "meanDim"):
            c = getattr(rt, op)(x["id"], d, False)
            o = getattr(orc, op)(ox["id"], d, False)
            assert_scaled(rt.toNumpy(c["id"]), orc.array(o["id"]), what=f"{op} {d}")
            free(rt, c)
        cv, ci = rt.maxDim(x["id"], d, False)
        ov, oi = orc.maxDim(ox["id"], d, False)
        assert np.array_equal(rt.toNumpy(cv["id"]), orc.array(ov["id"])), f"max values dim {d}"
        assert np.array_equal(rt.toNumpy(ci["id"]), orc.array(oi["id"])), f"max indices dim {d}"
        free(rt, cv, ci)
    for op in ("sum", "mean", "max"):
        c = getattr(rt, op)(x["id"])
        o = getattr(orc, op)(ox["id"])
        assert_scaled(rt.toNumpy(c["id"]), orc.array(o["id"]), what=op)
        free(rt, c)
    am = rt.argmax(x["id"])
    oam = orc.argmax(ox["id"])
    assert np.array_equal(rt.toNumpy(am["id"]), orc.array(oam["id"]))
    free(rt, x, am)


def test_batchnorm_train_256x128x56x56_fwd_bwd(cuda_rt, oracle_rt):
    rt, orc = cuda_rt, oracle_rt
    shp, C = [256, 128, 56, 56], 128
    rng = np.random.default_rng(12)
    gam, bet = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32), (0.1 * rng.standard_normal(C)).astype(np.float32)
    x, dy = randn(rt, shp, 401), randn(rt, shp, 402)
    g, b, rm, rv = dev_t(rt, gam), dev_t(rt, bet), dev_t(rt, np.zeros(C)), dev_t(rt, np.ones(C))
    y, mean, inv = rt.batchNormTrain(x["id"], g["id"], b["id"], rm["id"], rv["id"], 1e-5, 0.1)
    dx, dg, db = rt.batchNormBackward(dy["id"], x["id"], g["id"], mean["id"], inv["id"])
    ox, ody = orc_t(orc, host(rt, x)), orc_t(orc, host(rt, dy))
    og, ob, orm, orv = (orc_t(orc, a) for a in (gam, bet, np.zeros(C), np.ones(C)))
    oy, om, oi = orc.batchNormTrain(ox["id"], og["id"], ob["id"], orm["id"], orv["id"], 1e-5, 0.1)
    odx, odg, odb = orc.batchNormBackward(ody["id"], ox["id"], og["id"], om["id"], oi["id"])
    for c, o, nm in ((y, oy, "y"), (mean, om, "mean"), (inv, oi, "invstd"), (rm, orm, "running_mean"),
                     (rv, orv, "running_var"), (dx, odx, "dx"), (dg, odg, "dgamma"), (db, odb, "dbeta")):
        assert_scaled(rt.toNumpy(c["id"]), orc.array(o["id"]), what=nm)
    free(rt, x, dy, g, b, rm, rv, y, mean, inv, dx, dg, db)
    for h in (ox, ody, og, ob, orm, orv, oy, om, oi, odx, odg, odb):
        orc.destroy(h["id"])


# ---- dense contractions (configs: matmul, linear, conv) -----------------------------------------


@pytest.mark.parametrize("n", [512, 2048, 8192])
def test_matmul_square_sampled(cuda_rt, oracle_rt, n):
    rt, orc = cuda_rt, oracle_rt
    a, b = uniform(rt, [n, n], 500 + n), uniform(rt, [n, n], 501 + n)
    c = rt.matmul(a["id"], b["id"])
    A, B, Cd = host(rt, a), host(rt, b), host(rt, c)
    rng = np.random.default_rng(n)
    k = min(n, 96)
    rows, cols = np.sort(rng.choice(n, k, replace=False)), np.sort(rng.choice(n, k, replace=False))
    rows[0], cols[-1] = 0, n - 1  # the first row tile and the last column tile
    o = orc.matmul(orc_t(orc, A[rows])["id"], orc_t(orc, B[:, cols])["id"])
    assert_scaled(Cd[np.ix_(rows, cols)], orc.array(o["id"]).reshape(k, k), what=f"matmul {n}")
    free(rt, a, b, c)


def test_linear_16384x4096x11008_bias_sampled(cuda_rt, oracle_rt):
    rt, orc = cuda_rt, oracle_rt
    M, K, N = 16384, 4096, 11008
    x, w, b = uniform(rt, [M, K], 601), uniform(rt, [N, K], 602), uniform(rt, [N], 603)
    y = rt.linear(x["id"], w["id"], b["id"])
    assert y["shape"] == [M, N]
    X, W, Bv, Y = host(rt, x), host(rt, w), host(rt, b), host(rt, y)
    rng = np.random.default_rng(7)
    rows = np.sort(rng.choice(M, 64, replace=False))
    cols = np.sort(rng.choice(N, 64, replace=False))
    rows[-1], cols[-1] = M - 1, N - 1
    ow = orc.transpose2d(orc_t(orc, W[cols])["id"])
    o = orc.add(orc.matmul(orc_t(orc, X[rows])["id"], ow["id"])["id"], orc_t(orc, Bv[cols])["id"])
    assert_scaled(Y[np.ix_(rows, cols)], orc.array(o["id"]).reshape(64, 64), what="linear")
    free(rt, x, w, b, y)


CONV_CFGS = [
    # x shape, w shape, stride, padding
    ([128, 64, 56, 56], [64, 64, 3, 3], 1, 1),
    ([128, 3, 224, 224], [64, 3, 7, 7], 2, 3),
]


@pytest.mark.parametrize("xs,ws,st,pd", CONV_CFGS, ids=["3x3_64_56", "7x7s2_3_224"])
def test_conv2d_fwd_dgrad_wgrad_sampled(cuda_rt, oracle_rt, xs, ws, st, pd):
    """Forward and data gradient: whole sampled images (images are independent);
    weight gradient: sampled output channels over the whole batch."""
    rt, orc = cuda_rt, oracle_rt
    N, Cin, H, W = xs
    Cout, _, KH, KW = ws
    OH = (H + 2 * pd - KH) // st + 1
    OW = (W + 2 * pd - KW) // st + 1
    ys = [N, Cout, OH, OW]
    x = randn(rt, xs, 701)
    rt.setSeed(702)
    w = rt.normal(ws, "float32", 0.0, math.sqrt(2.0 / (Cin * KH * KW)))  # Kaiming-normal
    gy = randn(rt, ys, 703)
    bias = [0.01 * i for i in range(Cout)]
    y = rt.conv2d(x["id"], w["id"], bias, [st], [pd], [1], 1)
    dx = rt.conv2dInputBackward(gy["id"], w["id"], xs, ys, [st], [pd])
    dw = rt.conv2dWeightBackward(gy["id"], x["id"], ws, ys, xs, [st], [pd])
    assert y["shape"] == ys and dx["shape"] == xs and dw["shape"] == ws
    X, Wt, GY = host(rt, x), host(rt, w), host(rt, gy)
    Y, DX, DW = host(rt, y), host(rt, dx), host(rt, dw)
    imgs = [0, N - 1]
    ow = orc_t(orc, Wt)
    oy = orc.conv2d(orc_t(orc, X[imgs])["id"], ow["id"], bias, [st], [pd], [1], 1)
    assert_scaled(Y[imgs], orc.array(oy["id"]).reshape([2] + ys[1:]), what="conv fwd")
    odx = orc.conv2dInputBackward(orc_t(orc, GY[imgs])["id"], ow["id"], [2] + xs[1:], [2] + ys[1:], [st], [pd])
    assert_scaled(DX[imgs], orc.array(odx["id"]).reshape([2] + xs[1:]), what="conv dgrad")
    chans = [0, Cout // 2 + 1, Cout - 1]
    odw = orc.conv2dWeightBackward(orc_t(orc, GY[:, chans])["id"], orc_t(orc, X)["id"], [len(chans), Cin, KH, KW],
                                   [N, len(chans), OH, OW], xs, [st], [pd])
    ODW = orc.array(odw["id"]).reshape(len(chans), Cin, KH, KW).astype(np.float64)
    # Each weight-gradient value sums N*OH*OW = 0.4 M / 1.6 M products.  The
    # reference's sequential fp32 sum itself drifts from the exact value by
    # ~1e-5..1e-4 of the scale at this length, so the device result is held to
    # 1e-4 of the exact (float64) sum, and to the oracle within 1e-4 plus the
    # oracle's own distance from the exact sum.
    G = GY[:, chans].astype(np.float64)
    Xp = np.pad(X.astype(np.float64), ((0, 0), (0, 0), (pd, pd), (pd, pd)))
    exact = np.zeros((len(chans), Cin, KH, KW))
    for kh in range(KH):
        for kw in range(KW):
            xsl = Xp[:, :, kh:kh + st * (OH - 1) + 1:st, kw:kw + st * (OW - 1) + 1:st]
            exact[:, :, kh, kw] = np.einsum("nohw,nchw->oc", G, xsl, optimize=True)
    scale = float(np.max(np.abs(exact)))
    assert_scaled(DW[chans], exact, what="conv wgrad vs exact")
    orc_drift = float(np.max(np.abs(ODW - exact)))
    err = float(np.max(np.abs(DW[chans].astype(np.float64) - ODW)))
    assert err <= REL * scale + orc_drift, ("conv wgrad vs oracle", err, scale, orc_drift)
    free(rt, x, w, gy, y, dx, dw)


# ---- fused optimizer steps over the whole 64-tensor set (config: optimizer) ----------------------

SHAPES = [[4096, 4096], [4096], [1024, 4096], [4096, 1024]]


def _adam_scalars(step, lr=1e-3, b1=0.9, b2=0.999):
    return lr / (1.0 - b1 ** step), 1.0 / math.sqrt(1.0 - b2 ** step)


@pytest.mark.parametrize("kind", ["adamw", "sgd_nesterov"])
def test_optimizer_step_64_tensors_bit_exact(cuda_rt, oracle_rt, kind):
    rt, orc = cuda_rt, oracle_rt
    n = 64
    rt.setSeed(811)
    P = [rt.normal(SHAPES[i % 4], "float32", 0.0, 0.02) for i in range(n)]
    S0 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(n)]
    S1 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(n)] if kind == "adamw" else None
    rng = np.random.default_rng(5)
    sample = [4 * int(rng.integers(0, 16)) + j for j in range(4)]  # one tensor of each shape
    op = {i: orc_t(orc, host(rt, P[i])) for i in sample}
    os0 = {i: orc_t(orc, np.zeros(P[i]["shape"], np.float32)) for i in sample}
    os1 = {i: orc_t(orc, np.zeros(P[i]["shape"], np.float32)) for i in sample}
    ids = lambda hs: [h["id"] for h in hs]  # noqa: E731
    for step in (1, 2, 3):
        rt.setSeed(900 + step)
        G = [rt.normal(SHAPES[i % 4], "float32", 0.0, 1e-3) for i in range(n)]
        og = {i: orc_t(orc, host(rt, G[i])) for i in sample}
        if kind == "adamw":
            ss, isb = _adam_scalars(step)
            rt.adamWStepMulti(ids(P), ids(G), ids(S0), ids(S1), 1e-3, 0.9, 0.999, 1e-8, 0.01, ss, isb)
            orc.adamWStepMulti([op[i]["id"] for i in sample], [og[i]["id"] for i in sample],
                               [os0[i]["id"] for i in sample], [os1[i]["id"] for i in sample],
                               1e-3, 0.9, 0.999, 1e-8, 0.01, ss, isb)
        else:
            rt.sgdStepMulti(ids(P), ids(G), ids(S0), 1e-3, 0.9, 0.0, 0.0, True)
            orc.sgdStepMulti([op[i]["id"] for i in sample], [og[i]["id"] for i in sample],
                             [os0[i]["id"] for i in sample], 1e-3, 0.9, 0.0, 0.0, True)
        free(rt, *G)
        for h in og.values():
            orc.destroy(h["id"])
    for i in sample:
        assert np.array_equal(rt.toNumpy(P[i]["id"]), orc.array(op[i]["id"])), f"param {i}"
        assert np.array_equal(rt.toNumpy(S0[i]["id"]), orc.array(os0[i]["id"])), f"state0 {i}"
        if kind == "adamw":
            assert np.array_equal(rt.toNumpy(S1[i]["id"]), orc.array(os1[i]["id"])), f"state1 {i}"
    free(rt, *P, *S0, *(S1 or []))
    for d in (op, os0, os1):
        for h in d.values():
            orc.destroy(h["id"])
