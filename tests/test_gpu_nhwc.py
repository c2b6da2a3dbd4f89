"""Channels-last norm / pool / bias kernels (tpk_*_nhwc) against their NCHW
counterparts on the same values: BatchNorm train forward (+ReLU, running
statistics) and backward (+ReLU mask), the per-channel sum, 2x2 max-pool
values, indices (bit-exact) and backward, and the NCHW -> channels-last
conversion."""
import ctypes

import numpy as np
import pytest

from test_gpu_tma import dev, empty, free, nchw, nhwc, read

pytestmark = pytest.mark.gpu
vp = ctypes.c_void_p


def close(got, ref, rel):
    scale = max(1e-30, float(np.max(np.abs(ref))))
    assert float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64)))) <= rel * scale


@pytest.mark.parametrize("n,c,hw", [(4, 64, 32), (16, 128, 8), (8, 512, 2), (3, 36, 5)])
def test_bn_nhwc_matches_nchw(cuda_rt, n, c, hw):
    rt, L = cuda_rt, cuda_rt.lib
    rng = np.random.default_rng(n * c + hw)
    x = (rng.standard_normal((n, c, hw, hw)) * 2 + 0.5).astype(np.float32)
    dy = rng.standard_normal((n, c, hw, hw)).astype(np.float32)
    gam = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    bet = (0.1 * rng.standard_normal(c)).astype(np.float32)
    P, S = n * hw * hw, hw * hw
    outs = {}
    for lay in ("nchw", "nhwc"):
        t = (lambda a: a) if lay == "nchw" else nhwc
        px, pdy, pg, pb = dev(rt, t(x)), dev(rt, t(dy)), dev(rt, gam), dev(rt, bet)
        rm, rv = dev(rt, np.zeros(c)), dev(rt, np.ones(c))
        y, mean, inv, dx, dg, db, cs = (empty(rt, k) for k in (x.size, c, c, x.size, c, c, c))
        if lay == "nchw":
            assert L.tpk_bn_train(vp(px), vp(pg), vp(pb), vp(rm), vp(rv), vp(y), vp(mean), vp(inv), n, c, S, 1e-5,
                                  0.1, 1) == 0
            assert L.tpk_bn_backward(vp(pdy), vp(px), vp(y), vp(pg), vp(mean), vp(inv), vp(dx), vp(dg), vp(db), n,
                                     c, S) == 0
            assert L.tpk_channel_sum(vp(pdy), n, c, S, vp(cs)) == 0
            back = lambda p: read(rt, p, x.shape)  # noqa: E731
        else:
            assert L.tpk_bn_train_nhwc(vp(px), vp(pg), vp(pb), vp(rm), vp(rv), vp(y), vp(mean), vp(inv), P, c, 1e-5,
                                       0.1, 1) == 0
            dxs = empty(rt, c)
            assert L.tpk_bn_backward_nhwc(vp(pdy), vp(px), vp(y), vp(pg), vp(mean), vp(inv), vp(dx), vp(dg), vp(db),
                                          vp(dxs), P, c) == 0
            assert L.tpk_channel_sum_nhwc(vp(pdy), P, c, vp(cs)) == 0
            dxn = nchw(read(rt, dx, (n, hw, hw, c)))
            # the fused per-channel sum of dx equals a separate sum of dx
            got_sum = read(rt, dxs, (c,)).astype(np.float64)
            want_sum = dxn.astype(np.float64).sum(axis=(0, 2, 3))
            assert np.max(np.abs(got_sum - want_sum)) <= 1e-4 * max(1.0, float(np.max(np.abs(dxn)))) * 8
            free(rt, dxs)
            back = lambda p: nchw(read(rt, p, (n, hw, hw, c)))  # noqa: E731
        outs[lay] = {"y": back(y), "dx": back(dx), "mean": read(rt, mean, (c,)), "inv": read(rt, inv, (c,)),
                     "rm": read(rt, rm, (c,)), "rv": read(rt, rv, (c,)), "dg": read(rt, dg, (c,)),
                     "db": read(rt, db, (c,)), "cs": read(rt, cs, (c,))}
        free(rt, px, pdy, pg, pb, rm, rv, y, mean, inv, dx, dg, db, cs)
    a, b = outs["nchw"], outs["nhwc"]
    for k in a:
        close(b[k], a[k], 1e-5)


@pytest.mark.parametrize("n,c,hw", [(4, 64, 32), (16, 512, 2), (2, 12, 6)])
def test_maxpool_nhwc_matches_nchw(cuda_rt, n, c, hw):
    rt, L = cuda_rt, cuda_rt.lib
    rng = np.random.default_rng(n + c + hw)
    x = rng.standard_normal((n, c, hw, hw)).astype(np.float32)
    x[0, 0, :2, :2] = 1.5  # a tie: the first maximum in row-major window order wins
    oh = hw // 2
    gy = rng.standard_normal((n, c, oh, oh)).astype(np.float32)
    px, pxn, pgy, pgyn = dev(rt, x), dev(rt, nhwc(x)), dev(rt, gy), dev(rt, nhwc(gy))
    y0, y1, i0, i1, gx0, gx1 = (empty(rt, k) for k in (gy.size, gy.size, gy.size, gy.size, x.size, x.size))
    assert L.tpk_maxpool_fwd(vp(px), vp(y0), vp(i0), n, c, hw, hw, 2, 2, 0) == 0
    assert L.tpk_maxpool_bwd(vp(pgy), vp(i0), vp(gx0), n, c, hw, hw, 2, 2, 0) == 0
    assert L.tpk_maxpool2x2_nhwc_fwd(vp(pxn), vp(y1), vp(i1), n, hw, hw, c) == 0
    assert L.tpk_maxpool2x2_nhwc_bwd(vp(pgyn), vp(i1), vp(gx1), n, hw, hw, c) == 0

    def ints(p, shape):
        out = np.zeros(int(np.prod(shape)), np.int32)
        assert L.tp_memcpy_d2h(out.ctypes.data_as(vp), vp(p), out.nbytes) == 0
        return out.reshape(shape)

    assert np.array_equal(read(rt, y0, gy.shape), nchw(read(rt, y1, (n, oh, oh, c))))
    assert np.array_equal(ints(i0, gy.shape), nchw(ints(i1, (n, oh, oh, c))))
    assert np.array_equal(read(rt, gx0, x.shape), nchw(read(rt, gx1, (n, hw, hw, c))))
    free(rt, px, pxn, pgy, pgyn, y0, y1, i0, i1, gx0, gx1)


def ints(rt, p, shape):
    out = np.zeros(int(np.prod(shape)), np.int32)
    assert rt.lib.tp_memcpy_d2h(out.ctypes.data_as(vp), vp(p), out.nbytes) == 0
    return out.reshape(shape)


@pytest.mark.parametrize("relu", [1, 0])
@pytest.mark.parametrize("n,c,h,w", [(4, 64, 32, 32), (3, 36, 6, 10), (2, 512, 4, 4), (5, 16, 14, 2)])
def test_bn_pool_fused_matches_unfused(cuda_rt, n, c, h, w, relu):
    """BN train + ReLU + 2x2 pool in one pass against tpk_bn_train_nhwc then
    tpk_maxpool2x2_nhwc_fwd (bit-exact: values, indices, statistics, the
    optional full-size output); the fused backward (pool gradient read in
    place, ReLU mask from the BN input) against tpk_maxpool2x2_nhwc_bwd then
    tpk_bn_backward_nhwc (masked by the stored activation)."""
    rt, L = cuda_rt, cuda_rt.lib
    rng = np.random.default_rng(n * c + h * w + relu)
    x = (rng.standard_normal((n, h, w, c)) * 2 + 0.3).astype(np.float32)
    x[0, 0, 0, :] = x[0, 0, 1, :]  # ties inside a window: the first maximum wins
    gam = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    bet = (0.2 * rng.standard_normal(c)).astype(np.float32)
    oh, ow = h // 2, w // 2
    gp = rng.standard_normal((n, oh, ow, c)).astype(np.float32)
    P, Q = n * h * w, n * oh * ow
    px, pg, pb, pgp = dev(rt, x), dev(rt, gam), dev(rt, bet), dev(rt, gp)
    out = {}
    for mode in ("unfused", "fused"):
        rm, rv = dev(rt, np.full(c, 0.1)), dev(rt, np.full(c, 0.9))
        a, y, idx, mean, inv = empty(rt, P * c), empty(rt, Q * c), empty(rt, Q * c), empty(rt, c), empty(rt, c)
        dx, dg, db, dxs, da = empty(rt, P * c), empty(rt, c), empty(rt, c), empty(rt, c), empty(rt, P * c)
        if mode == "unfused":
            assert L.tpk_bn_train_nhwc(vp(px), vp(pg), vp(pb), vp(rm), vp(rv), vp(a), vp(mean), vp(inv), P, c,
                                       1e-5, 0.1, relu) == 0
            assert L.tpk_maxpool2x2_nhwc_fwd(vp(a), vp(y), vp(idx), n, h, w, c) == 0
            assert L.tpk_maxpool2x2_nhwc_bwd(vp(pgp), vp(idx), vp(da), n, h, w, c) == 0
            assert L.tpk_bn_backward_nhwc(vp(da), vp(px), vp(a) if relu else None, vp(pg), vp(mean), vp(inv),
                                          vp(dx), vp(dg), vp(db), vp(dxs), P, c) == 0
        else:
            assert L.tpk_bn_train_pool_nhwc(vp(px), vp(pg), vp(pb), vp(rm), vp(rv), vp(y), vp(idx), vp(a),
                                            vp(mean), vp(inv), n, h, w, c, 1e-5, 0.1, relu) == 0
            assert L.tpk_bn_backward_fused_nhwc(vp(pgp), vp(idx), vp(px), vp(pg), vp(pb), vp(mean), vp(inv),
                                                vp(dx), vp(dg), vp(db), vp(dxs), n, h, w, c, relu) == 0
        out[mode] = {"a": read(rt, a, (P * c,)), "y": read(rt, y, (Q * c,)), "idx": ints(rt, idx, (Q * c,)),
                     "mean": read(rt, mean, (c,)), "inv": read(rt, inv, (c,)), "rm": read(rt, rm, (c,)),
                     "rv": read(rt, rv, (c,)), "dx": read(rt, dx, (P * c,)), "dg": read(rt, dg, (c,)),
                     "db": read(rt, db, (c,)), "dxs": read(rt, dxs, (c,))}
        free(rt, rm, rv, a, y, idx, mean, inv, dx, dg, db, dxs, da)
    free(rt, px, pg, pb, pgp)
    u, f = out["unfused"], out["fused"]
    for k in ("a", "y", "idx", "mean", "inv", "rm", "rv"):
        assert np.array_equal(u[k], f[k]), k
    # the backward sums run over windows instead of pixel rows: same terms, another order
    for k in ("dx", "dg", "db"):
        close(f[k], u[k], 1e-5)
    close(f["dxs"], u["dxs"], 1e-4)


@pytest.mark.parametrize("n,c,hw", [(4, 64, 16), (2, 512, 2)])
def test_bn_backward_relu_from_input(cuda_rt, n, c, hw):
    """tpk_bn_backward_fused_nhwc without a pool: the ReLU mask recomputed from
    the BN input equals the one read from the stored activation, so every
    output is bit-identical to tpk_bn_backward_nhwc's."""
    rt, L = cuda_rt, cuda_rt.lib
    rng = np.random.default_rng(c + hw)
    x = (rng.standard_normal((n, hw, hw, c)) + 0.2).astype(np.float32)
    dy = rng.standard_normal((n, hw, hw, c)).astype(np.float32)
    gam = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    bet = (0.3 * rng.standard_normal(c)).astype(np.float32)
    P = n * hw * hw
    px, pdy, pg, pb = dev(rt, x), dev(rt, dy), dev(rt, gam), dev(rt, bet)
    rm, rv, a, mean, inv = empty(rt, c), empty(rt, c), empty(rt, P * c), empty(rt, c), empty(rt, c)
    assert L.tpk_bn_train_nhwc(vp(px), vp(pg), vp(pb), vp(rm), vp(rv), vp(a), vp(mean), vp(inv), P, c, 1e-5, 0.1,
                               1) == 0
    res = []
    for fused in (False, True):
        dx, dg, db, dxs = empty(rt, P * c), empty(rt, c), empty(rt, c), empty(rt, c)
        if fused:
            assert L.tpk_bn_backward_fused_nhwc(vp(pdy), None, vp(px), vp(pg), vp(pb), vp(mean), vp(inv), vp(dx),
                                                vp(dg), vp(db), vp(dxs), n, hw, hw, c, 1) == 0
        else:
            assert L.tpk_bn_backward_nhwc(vp(pdy), vp(px), vp(a), vp(pg), vp(mean), vp(inv), vp(dx), vp(dg),
                                          vp(db), vp(dxs), P, c) == 0
        res.append([read(rt, p, (k,)) for p, k in ((dx, P * c), (dg, c), (db, c), (dxs, c))])
        free(rt, dx, dg, db, dxs)
    free(rt, px, pdy, pg, pb, rm, rv, a, mean, inv)
    for u, f in zip(*res):
        assert np.array_equal(u, f)


def test_nchw_to_nhwc_padded(cuda_rt):
    rt, L = cuda_rt, cuda_rt.lib
    x = np.random.default_rng(0).standard_normal((5, 3, 7, 9)).astype(np.float32)
    px, py = dev(rt, x), empty(rt, 5 * 7 * 9 * 32)
    assert L.tpk_nchw_to_nhwc(vp(px), vp(py), 5, 3, 7, 9, 32) == 0
    got = read(rt, py, (5, 7, 9, 32))
    assert np.array_equal(got[..., :3], nhwc(x)) and not np.any(got[..., 3:])
    free(rt, px, py)
