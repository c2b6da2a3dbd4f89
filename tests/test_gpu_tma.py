"""TMA-fed tensor-core GEMM (tp_gemm_tma.cuh) and the channels-last
convolutions built on it (tpk_conv2d_*_nhwc).

The TMA kernel splits operands and issues MMAs exactly like the gather
kernel, so for the same tile shape and split-K the two must agree bit for bit:
every dense case compares engine 0 (TMA where the operands allow) with engine 2
(gather only) for exact equality, and both against a float64 product.  The
channels-last convolutions are checked against the NCHW kernels (themselves
checked against the oracle) after a layout transpose, and directly against the
oracle for one shape per pass."""
import ctypes

import numpy as np
import pytest

from test_gpu_gemm_paths import status

pytestmark = pytest.mark.gpu


def dev(rt, arr):
    arr = np.ascontiguousarray(arr, np.float32)
    p = ctypes.c_void_p()
    assert rt.lib.tp_alloc(max(4, arr.nbytes), ctypes.byref(p)) == 0
    if arr.size:
        assert rt.lib.tp_memcpy_h2d(p, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes) == 0
    return p.value


def empty(rt, n):
    p = ctypes.c_void_p()
    assert rt.lib.tp_alloc(max(4, n * 4), ctypes.byref(p)) == 0
    return p.value


def read(rt, p, shape):
    out = np.zeros(int(np.prod(shape)), np.float32)
    assert rt.lib.tp_memcpy_d2h(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(p), out.nbytes) == 0
    return out.reshape(shape)


def free(rt, *ps):
    for p in ps:
        rt.lib.tp_free(ctypes.c_void_p(p))


@pytest.fixture
def engine(cuda_rt):
    def set_path(p):
        assert cuda_rt.lib.tp_set_gemm_path(p) == 0
    yield set_path
    cuda_rt.lib.tp_set_gemm_path(0)


def close64(got, ref, rel=1e-4):
    scale = max(1e-30, float(np.max(np.abs(ref))))
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    assert err <= rel * scale, (err, scale)


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (200, 52, 68), (64, 16, 1000), (512, 384, 4096),
                                   (1000, 300, 36), (300, 1000, 2048), (96, 40, 8), (384, 96, 160),
                                   (2048, 512, 1024)])
@pytest.mark.parametrize("a_t", [0, 1])
@pytest.mark.parametrize("b_t", [0, 1])
def test_gemm_tma_bitwise_equals_gather(cuda_rt, engine, M, N, K, a_t, b_t):
    rt = cuda_rt
    rng = np.random.default_rng(M * 7 + N * 3 + K + 2 * a_t + b_t)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    pa = dev(rt, A.T if a_t else A)
    pb = dev(rt, B.T if b_t else B)
    pbias = dev(rt, bias)
    outs = []
    # 3: single-CTA TMA tiles, bit-identical to the gather kernel (same tiles and
    # split); 0: the default choice; 4: CTA pairs wherever they fit
    for path in (3, 2, 0, 4):
        engine(path)
        pc = empty(rt, M * N)
        assert rt.lib.tpk_gemm(ctypes.c_void_p(pa), a_t, ctypes.c_void_p(pb), b_t, ctypes.c_void_p(pc), M, N, K,
                               ctypes.c_void_p(pbias)) == 0
        outs.append(read(rt, pc, (M, N)))
        free(rt, pc)
        assert status(rt) == 0
    free(rt, pa, pb, pbias)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    ref = A.astype(np.float64) @ B.astype(np.float64) + bias
    close64(outs[0], ref)
    close64(outs[2], ref)
    close64(outs[3], ref)


def test_matmul_handle_tma_long_k(cuda_rt, oracle_rt):
    """K = 8192 through the handle API on the TMA kernel: fp32 accuracy holds."""
    from test_gpu_dense import close_scaled
    from test_gpu_ops import both
    rng = np.random.default_rng(5)
    ca, oa = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (256, 8192)))
    cb, ob = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (8192, 256)))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.matmul(ca["id"], cb["id"]), oracle_rt.matmul(oa["id"], ob["id"]),
                 rel=2e-5)
    assert status(cuda_rt) == 0


# (Cin, Cout, H=W) of every VGG-11-BN conv (the first with its input padded to 4
# channels too), plus shapes off the TMA kernel and off whole-row pixel tiles
NHWC_SHAPES = [(3, 64, 32), (4, 64, 32), (4, 16, 7), (64, 128, 16), (128, 256, 8), (256, 256, 8), (256, 512, 4),
               (512, 512, 4), (512, 512, 2), (32, 64, 6), (48, 96, 8),
               # pixel grids that 128 / 32 pixel runs do not tile: rectangle tiles
               (64, 64, 14), (32, 64, 7), (64, 64, 20)]


def nchw(a):
    return np.ascontiguousarray(a.transpose(0, 3, 1, 2))


def nhwc(a):
    return np.ascontiguousarray(a.transpose(0, 2, 3, 1))


@pytest.mark.parametrize("cin,cout,hw", NHWC_SHAPES)
@pytest.mark.parametrize("batch", [4, 16])
@pytest.mark.parametrize("nhwc_path", [0, 4], ids=["default", "cta_pairs"])
def test_conv_nhwc_matches_nchw(cuda_rt, engine, cin, cout, hw, batch, nhwc_path):
    rt = cuda_rt
    rng = np.random.default_rng(cin + 3 * cout + hw + batch)
    x = rng.standard_normal((batch, cin, hw, hw)).astype(np.float32)
    w = (rng.standard_normal((cout, cin, 3, 3)) * 0.05).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    dy = rng.standard_normal((batch, cout, hw, hw)).astype(np.float32)
    px, pxn, pw, pb, pdy, pdyn = dev(rt, x), dev(rt, nhwc(x)), dev(rt, w), dev(rt, b), dev(rt, dy), dev(rt, nhwc(dy))
    n_y, n_x, n_w = batch * cout * hw * hw, batch * cin * hw * hw, cout * cin * 9
    y0, y1, dx0, dx1, dw0, dw1 = (empty(rt, n) for n in (n_y, n_y, n_x, n_x, n_w, n_w))
    L = rt.lib
    vp = ctypes.c_void_p
    engine(2)  # NCHW reference side on the gather kernels
    assert L.tpk_conv2d_fwd(vp(px), vp(pw), vp(pb), vp(y0), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1, 1) == 0
    assert L.tpk_conv2d_dgrad(vp(pdy), vp(pw), vp(dx0), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1, 1) == 0
    assert L.tpk_conv2d_wgrad(vp(pdy), vp(px), vp(dw0), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1, 1) == 0
    engine(nhwc_path)
    assert L.tpk_conv2d_fwd_nhwc(vp(pxn), vp(pw), vp(pb), vp(y1), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert L.tpk_conv2d_dgrad_nhwc(vp(pdyn), vp(pw), vp(dx1), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert L.tpk_conv2d_wgrad_nhwc(vp(pdyn), vp(pxn), vp(dw1), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert status(rt) == 0
    ref_y = read(rt, y0, (batch, cout, hw, hw))
    got_y = nchw(read(rt, y1, (batch, hw, hw, cout)))
    ref_dx = read(rt, dx0, (batch, cin, hw, hw))
    got_dx = nchw(read(rt, dx1, (batch, hw, hw, cin)))
    ref_dw = read(rt, dw0, (cout, cin, 3, 3))
    got_dw = read(rt, dw1, (cout, cin, 3, 3))
    free(rt, px, pxn, pw, pb, pdy, pdyn, y0, y1, dx0, dx1, dw0, dw1)
    # two fp32 summation orders of the same products (different tile shapes and
    # split-K plans): the parity bar, 1e-4 of the output scale
    for got, ref in ((got_y, ref_y), (got_dx, ref_dx), (got_dw, ref_dw)):
        close64(got, ref.astype(np.float64), rel=1e-4)


@pytest.mark.parametrize("cin,cout,hw,batch", [(64, 128, 16, 4), (256, 256, 8, 8), (3, 64, 32, 2), (4, 64, 32, 2)])
def test_conv_nhwc_against_oracle(cuda_rt, oracle_rt, cin, cout, hw, batch):
    rt, orc = cuda_rt, oracle_rt
    rng = np.random.default_rng(cin * cout + hw)
    x = rng.standard_normal((batch, cin, hw, hw)).astype(np.float32)
    w = (rng.standard_normal((cout, cin, 3, 3)) * 0.05).astype(np.float32)
    dy = rng.standard_normal((batch, cout, hw, hw)).astype(np.float32)
    T = lambda a: orc.tensorFromData(a.ravel().tolist(), list(a.shape), "float32")["id"]  # noqa: E731
    ox, ow, ody = T(x), T(w), T(dy)
    ref_y = np.asarray(orc.toList(orc.conv2d(ox, ow, None, [1], [1], [1], 1)["id"]), np.float64).reshape(dy.shape)
    ref_dx = np.asarray(orc.toList(orc.conv2dInputBackward(ody, ow, list(x.shape), list(dy.shape), [1], [1])["id"]),
                        np.float64).reshape(x.shape)
    ref_dw = np.asarray(orc.toList(orc.conv2dWeightBackward(ody, ox, list(w.shape), list(dy.shape), list(x.shape),
                                                            [1], [1])["id"]), np.float64).reshape(w.shape)
    pxn, pw, pdyn = dev(rt, nhwc(x)), dev(rt, w), dev(rt, nhwc(dy))
    y, dx, dw = empty(rt, dy.size), empty(rt, x.size), empty(rt, w.size)
    vp = ctypes.c_void_p
    L = rt.lib
    assert L.tpk_conv2d_fwd_nhwc(vp(pxn), vp(pw), None, vp(y), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert L.tpk_conv2d_dgrad_nhwc(vp(pdyn), vp(pw), vp(dx), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert L.tpk_conv2d_wgrad_nhwc(vp(pdyn), vp(pxn), vp(dw), batch, cin, hw, hw, cout, 3, 3, 1, 1, 0) == 0
    assert status(rt) == 0
    close64(nchw(read(rt, y, (batch, hw, hw, cout))), ref_y)
    close64(nchw(read(rt, dx, (batch, hw, hw, cin))), ref_dx)
    close64(read(rt, dw, w.shape), ref_dw)
    free(rt, pxn, pw, pdyn, y, dx, dw)


@pytest.mark.parametrize("cin,cout,hw,batch", [(64, 128, 16, 4), (256, 256, 8, 8), (512, 512, 2, 8), (32, 64, 20, 2),
                                               (48, 96, 8, 4)])
@pytest.mark.parametrize("nhwc_path", [0, 4], ids=["default", "cta_pairs"])
def test_conv_nhwc_packed_filters(cuda_rt, engine, cin, cout, hw, batch, nhwc_path):
    """Filters stored [Cout][KH][KW][Cin] (filter_layout 1) give the same
    forward, data gradient and (permuted) weight gradient as the reference
    layout."""
    rt, L, vp = cuda_rt, cuda_rt.lib, ctypes.c_void_p
    engine(nhwc_path)
    rng = np.random.default_rng(cin + cout + hw + batch + 7)
    x = rng.standard_normal((batch, hw, hw, cin)).astype(np.float32)
    w = (rng.standard_normal((cout, cin, 3, 3)) * 0.05).astype(np.float32)
    wk = np.ascontiguousarray(w.transpose(0, 2, 3, 1))
    b = rng.standard_normal(cout).astype(np.float32)
    dy = rng.standard_normal((batch, hw, hw, cout)).astype(np.float32)
    px, pw, pwk, pb, pdy = dev(rt, x), dev(rt, w), dev(rt, wk), dev(rt, b), dev(rt, dy)
    outs = []
    for lay, pw_ in ((0, pw), (1, pwk)):
        y, dx, dw = empty(rt, dy.size), empty(rt, x.size), empty(rt, w.size)
        assert L.tpk_conv2d_fwd_nhwc(vp(px), vp(pw_), vp(pb), vp(y), batch, cin, hw, hw, cout, 3, 3, 1, 1, lay) == 0
        assert L.tpk_conv2d_dgrad_nhwc(vp(pdy), vp(pw_), vp(dx), batch, cin, hw, hw, cout, 3, 3, 1, 1, lay) == 0
        assert L.tpk_conv2d_wgrad_nhwc(vp(pdy), vp(px), vp(dw), batch, cin, hw, hw, cout, 3, 3, 1, 1, lay) == 0
        g = read(rt, dw, (cout, 3, 3, cin)).transpose(0, 3, 1, 2) if lay else read(rt, dw, w.shape)
        outs.append((read(rt, y, dy.shape), read(rt, dx, x.shape), np.ascontiguousarray(g)))
        free(rt, y, dx, dw)
    assert status(rt) == 0
    free(rt, px, pw, pwk, pb, pdy)
    for a, c in zip(outs[0], outs[1]):
        close64(c, a.astype(np.float64), rel=1e-5)


@pytest.mark.parametrize("cin,cout,hw,batch", [(64, 128, 16, 4), (256, 512, 4, 8), (128, 256, 8, 2)])
def test_conv_nhwc_filter_lo_entries(cuda_rt, cin, cout, hw, batch):
    """The forward / data-gradient entries that take the filters' tf32 low
    parts (tpk_tf32_lo of the filters) give the same bits as the entries that
    split them per call."""
    rt, L, vp = cuda_rt, cuda_rt.lib, ctypes.c_void_p
    rng = np.random.default_rng(cin + cout + batch)
    x = rng.standard_normal((batch, hw, hw, cin)).astype(np.float32)
    wk = (rng.standard_normal((cout, 3, 3, cin)) * 0.05).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    dy = rng.standard_normal((batch, hw, hw, cout)).astype(np.float32)
    px, pw, pb, pdy, plo = dev(rt, x), dev(rt, wk), dev(rt, b), dev(rt, dy), empty(rt, wk.size)
    assert L.tpk_tf32_lo(vp(pw), vp(plo), wk.size) == 0
    lo = read(rt, plo, wk.shape).astype(np.float64)
    hi = (wk.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32).astype(np.float64)
    assert np.array_equal(lo, wk.astype(np.float64) - hi)
    outs = []
    for use_lo in (False, True):
        y, dx = empty(rt, dy.size), empty(rt, x.size)
        if use_lo:
            assert L.tpk_conv2d_fwd_nhwc_lo(vp(px), vp(pw), vp(plo), vp(pb), vp(y), batch, cin, hw, hw, cout, 3, 3, 1,
                                            1, 1) == 0
            assert L.tpk_conv2d_dgrad_nhwc_lo(vp(pdy), vp(pw), vp(plo), vp(dx), batch, cin, hw, hw, cout, 3, 3, 1, 1,
                                              1) == 0
        else:
            assert L.tpk_conv2d_fwd_nhwc(vp(px), vp(pw), vp(pb), vp(y), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1) == 0
            assert L.tpk_conv2d_dgrad_nhwc(vp(pdy), vp(pw), vp(dx), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1) == 0
        outs.append((read(rt, y, dy.shape), read(rt, dx, x.shape)))
        free(rt, y, dx)
    assert status(rt) == 0
    free(rt, px, pw, pb, pdy, plo)
    for a, c in zip(outs[0], outs[1]):
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def test_sgd_group_writes_low_parts(cuda_rt):
    """An SGD group made with lo pointers updates params and momentum exactly as
    one without, and leaves each updated parameter's tf32 low parts in lo."""
    rt, L, vp = cuda_rt, cuda_rt.lib, ctypes.c_void_p
    rng = np.random.default_rng(3)
    sizes = [4096 * 3 + 7, 1000, 64]
    res = []
    for with_lo in (False, True):
        P = [dev(rt, rng.standard_normal(n) * 0.1) if not res else dev(rt, res[0]["p0"][i]) for i, n in enumerate(sizes)]
        if not res:
            p0 = [read(rt, p, (n,)) for p, n in zip(P, sizes)]
        G = [dev(rt, np.full(n, 0.01 * (i + 1), np.float32)) for i, n in enumerate(sizes)]
        Mo = [dev(rt, np.zeros(n, np.float32)) for n in sizes]
        LO = [empty(rt, n) for n in sizes]
        arr = lambda ps: (ctypes.c_void_p * len(ps))(*ps)  # noqa: E731
        numels = (ctypes.c_int64 * len(sizes))(*sizes)
        g = ctypes.c_int64(0)
        lo_rows = (ctypes.c_void_p * len(sizes))(LO[0], None, LO[2]) if with_lo else None
        assert L.tpk_group_create_lo(len(sizes), arr(P), arr(G), arr(Mo), None, lo_rows, numels, ctypes.byref(g)) == 0
        for _ in range(2):
            assert L.tpk_sgd_group(g.value, 0.05, 0.9, 5e-4, 0.0, 0, 0.5) == 0
        out = {"p": [read(rt, p, (n,)) for p, n in zip(P, sizes)], "m": [read(rt, m, (n,)) for m, n in zip(Mo, sizes)],
               "lo": [read(rt, q, (n,)) for q, n in zip(LO, sizes)]}
        if not res:
            out["p0"] = p0
        res.append(out)
        assert L.tpk_group_destroy(g.value) == 0
        free(rt, *P, *G, *Mo, *LO)
    a, c = res
    for i in range(len(sizes)):
        assert np.array_equal(a["p"][i], c["p"][i]) and np.array_equal(a["m"][i], c["m"][i])
    for i in (0, 2):
        p = c["p"][i]
        hi = (p.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
        assert np.array_equal(c["lo"][i], p - hi)


@pytest.mark.parametrize("cin,cout,hw,batch", [(64, 128, 16, 16), (128, 256, 8, 16), (128, 128, 12, 8)])
def test_conv_nhwc_two_ctas_per_sm_bitwise(cuda_rt, cin, cout, hw, batch):
    """128-column tiles on the 2-stage ring, two CTAs per SM (tp_set_gemm_twocta 2),
    against the 4-stage, one-per-SM kernel (0): the same split and MMA sequence,
    so the same bits for the forward, data and weight gradients."""
    rt = cuda_rt
    rng = np.random.default_rng(cin + cout + hw)
    x = rng.standard_normal((batch, hw, hw, cin)).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, cin)) * 0.05).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    dy = rng.standard_normal((batch, hw, hw, cout)).astype(np.float32)
    px, pw, pb, pdy = dev(rt, x), dev(rt, w), dev(rt, b), dev(rt, dy)
    vp = ctypes.c_void_p
    L = rt.lib
    outs = {}
    try:
        for mode in (0, 2):
            assert L.tp_set_gemm_twocta(mode) == 0
            y, dx, dw = empty(rt, x.size // cin * cout), empty(rt, x.size), empty(rt, w.size)
            assert L.tpk_conv2d_fwd_nhwc(vp(px), vp(pw), vp(pb), vp(y), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1) == 0
            assert L.tpk_conv2d_dgrad_nhwc(vp(pdy), vp(pw), vp(dx), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1) == 0
            assert L.tpk_conv2d_wgrad_nhwc(vp(pdy), vp(px), vp(dw), batch, cin, hw, hw, cout, 3, 3, 1, 1, 1) == 0
            assert status(rt) == 0
            outs[mode] = [read(rt, y, (x.size // cin * cout,)), read(rt, dx, (x.size,)), read(rt, dw, (w.size,))]
            free(rt, y, dx, dw)
    finally:
        assert L.tp_set_gemm_twocta(1) == 0
        free(rt, px, pw, pb, pdy)
    for a, c in zip(outs[0], outs[2]):
        assert np.array_equal(a, c)
