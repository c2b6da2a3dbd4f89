"""CUDA runtime vs the CPU oracle, op by op, on seeded inputs.

Tolerances (the bar stated for this path): bit-exact for integer / index work
and for ops whose arithmetic is fully IEEE-specified (+ - * /, sqrt, max,
compare, copies, the optimizer steps, rand); 1e-6 relative for element-wise
transcendentals; 1e-4 relative for reductions, norms, matmul and conv.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 3, 4, 7, 1023, 4096, 65537]


def both(cuda_rt, oracle_rt, arr, dtype="float32"):
    arr = np.ascontiguousarray(arr, dtype=np.float32)
    shape = list(arr.shape)
    c = cuda_rt.tensorFromData(arr.ravel(), shape, dtype)
    o = oracle_rt.tensorFromData(arr.ravel().tolist(), shape, dtype)
    return c, o


def vals(rt, h):
    return np.asarray(rt.toList(h["id"]), dtype=np.float64)


def check(cuda_rt, oracle_rt, hc, ho, rtol=0.0, atol=0.0):
    assert hc["shape"] == ho["shape"], (hc, ho)
    assert hc["dtype"] == ho["dtype"], (hc, ho)
    a, b = vals(cuda_rt, hc), vals(oracle_rt, ho)
    if rtol == 0.0 and atol == 0.0:
        assert np.array_equal(a, b, equal_nan=True), np.max(np.abs(a - b)) if a.size else 0
    else:
        np.testing.assert_allclose(a, b, rtol=rtol, atol=atol)


@pytest.mark.parametrize("n", SIZES)
def test_rand_bit_exact_and_randn(cuda_rt, oracle_rt, n):
    cuda_rt.setSeed(1234)
    oracle_rt.setSeed(1234)
    check(cuda_rt, oracle_rt, cuda_rt.rand([n], "float32"), oracle_rt.rand([n], "float32"))
    check(cuda_rt, oracle_rt, cuda_rt.randn([n], "float32"), oracle_rt.randn([n], "float32"), rtol=2e-6, atol=2e-6)


def test_seed_counter_matches(cuda_rt, oracle_rt):
    cuda_rt.setSeed(42)
    oracle_rt.setSeed(42)
    for _ in range(3):
        check(cuda_rt, oracle_rt, cuda_rt.rand([5], "float32"), oracle_rt.rand([5], "float32"))


@pytest.mark.parametrize("dtype,value", [("float32", 2.5), ("int32", -3.7), ("bool", 2.0), ("uint8", -1.0)])
def test_full_coerces_by_dtype(cuda_rt, oracle_rt, dtype, value):
    check(cuda_rt, oracle_rt, cuda_rt.full([3, 5], value, dtype), oracle_rt.full([3, 5], value, dtype))


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "maximum", "minimum", "eq", "ne", "lt", "le", "gt",
                                "ge"])
@pytest.mark.parametrize("n", [1, 7, 4096, 65537])
def test_binary_same_shape_bit_exact(cuda_rt, oracle_rt, op, n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    b[::5] = a[::5]  # some ties for the comparisons
    ca, oa = both(cuda_rt, oracle_rt, a)
    cb, ob = both(cuda_rt, oracle_rt, b)
    check(cuda_rt, oracle_rt, getattr(cuda_rt, op)(ca["id"], cb["id"]), getattr(oracle_rt, op)(oa["id"], ob["id"]))


# the last six hit the 16-byte [R][N] kernel: a bias row, a per-row column, a
# scalar, a 3-D shape that merges to 2-D, the row operand on the left
@pytest.mark.parametrize("sa,sb", [([2, 3], [3]), ([4, 1], [1, 5]), ([2, 3, 4, 5], [1, 3, 1, 1]),
                                   ([6, 1, 5], [7, 1]), ([3, 4], [1]), ([1], [2, 3, 2]), ([8, 16, 4], [16, 1]),
                                   ([64, 1024], [1024]), ([37, 20], [37, 1]), ([1], [256, 8]), ([5, 8, 16], [8, 16]),
                                   ([12], [9, 12]), ([3, 4], [3, 1])])
@pytest.mark.parametrize("op", ["add", "mul", "sub", "div", "gt"])
def test_binary_broadcast_bit_exact(cuda_rt, oracle_rt, sa, sb, op):
    rng = np.random.default_rng(len(sa) * 10 + len(sb))
    ca, oa = both(cuda_rt, oracle_rt, rng.standard_normal(sa))
    cb, ob = both(cuda_rt, oracle_rt, rng.standard_normal(sb) + 0.5)
    check(cuda_rt, oracle_rt, getattr(cuda_rt, op)(ca["id"], cb["id"]), getattr(oracle_rt, op)(oa["id"], ob["id"]))


def test_broadcast_error_matches(cuda_rt, oracle_rt):
    ca, oa = both(cuda_rt, oracle_rt, np.zeros((2, 3)))
    cb, ob = both(cuda_rt, oracle_rt, np.zeros((4,)))
    with pytest.raises(RuntimeError, match="cannot be broadcast"):
        cuda_rt.add(ca["id"], cb["id"])
    with pytest.raises(RuntimeError, match="cannot be broadcast"):
        oracle_rt.add(oa["id"], ob["id"])


def test_pow_integer_and_fractional(cuda_rt, oracle_rt):
    rng = np.random.default_rng(3)
    x = rng.uniform(0.1, 3.0, 257).astype(np.float32)
    e = np.array([2.0, 3.0, -1.0, 0.5, 1.5, 2.0000001, 64.0, -2.0] * 32 + [2.0], np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    ce, oe = both(cuda_rt, oracle_rt, e)
    check(cuda_rt, oracle_rt, cuda_rt.pow(cx["id"], ce["id"]), oracle_rt.pow(ox["id"], oe["id"]), rtol=1e-6)
    # integer exponents take the exact squaring path
    two = np.full(257, 2.0, np.float32)
    c2, o2 = both(cuda_rt, oracle_rt, two)
    check(cuda_rt, oracle_rt, cuda_rt.pow(cx["id"], c2["id"]), oracle_rt.pow(ox["id"], o2["id"]))


@pytest.mark.parametrize("op,rtol", [("relu", 0), ("neg", 0), ("abs", 0), ("sqrt", 0), ("square", 0),
                                     ("reciprocal", 0), ("rsqrt", 1e-6), ("exp", 1e-6), ("log", 1e-6),
                                     ("sigmoid", 1e-6), ("tanh", 1e-6)])
@pytest.mark.parametrize("n", [0, 5, 4099])
def test_unary(cuda_rt, oracle_rt, op, rtol, n):
    rng = np.random.default_rng(7)
    x = rng.standard_normal(n).astype(np.float32)
    if op in ("sqrt", "rsqrt", "log"):
        x = np.abs(x) + 0.01
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, getattr(cuda_rt, op)(cx["id"]), getattr(oracle_rt, op)(ox["id"]), rtol=rtol,
          atol=1e-7 if rtol else 0.0)


def test_mul_scalar(cuda_rt, oracle_rt):
    x = np.linspace(-3, 3, 1001).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, cuda_rt.mulScalar(cx["id"], 0.3), oracle_rt.mulScalar(ox["id"], 0.3))


@pytest.mark.parametrize("shape,op,args", [
    ([2, 3, 4], "reshape", ([4, 6],)), ([2, 3, 4], "flatten", (1,)), ([2, 1, 4], "squeeze", ()),
    ([2, 1, 4], "squeeze", (1,)), ([2, 4], "unsqueeze", (1,)), ([33, 65], "transpose2d", ()),
    ([2, 3, 4], "transpose", (0, 2)), ([2, 3, 4, 5], "permute", ([3, 1, 0, 2],)), ([3, 1], "expand", ([2, 3, 4],)),
    ([1, 5], "expand", ([4, 5],)), ([130, 257], "transpose2d", ())])
def test_shape_ops_bit_exact(cuda_rt, oracle_rt, shape, op, args):
    x = np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape)
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, getattr(cuda_rt, op)(cx["id"], *args), getattr(oracle_rt, op)(ox["id"], *args))


@pytest.mark.parametrize("n", [1, 5, 256, 257, 100003, 4 * 1024 * 1024 + 3])
def test_reduce_all(cuda_rt, oracle_rt, n):
    rng = np.random.default_rng(n % 1000)
    x = rng.standard_normal(n).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    scale = float(np.abs(x).sum()) + 1.0
    for m in ("sum", "mean", "max"):
        hc, ho = getattr(cuda_rt, m)(cx["id"]), getattr(oracle_rt, m)(ox["id"])
        assert hc["shape"] == ho["shape"] == []
        a, b = vals(cuda_rt, hc)[0], vals(oracle_rt, ho)[0]
        if m == "max":
            assert a == b
        else:
            tol = 1e-6 * scale / (n if m == "mean" else 1)
            assert abs(a - b) <= tol, (m, a, b)


@pytest.mark.parametrize("shape,dim", [([7, 9], 0), ([7, 9], 1), ([7, 9], -1), ([3, 5, 6], 1), ([2, 3, 4, 5], 2),
                                       ([4, 2000], -1), ([3000, 70], 0), ([1, 1], 0), ([512, 600], 0)])
@pytest.mark.parametrize("keepdim", [False, True])
def test_reduce_dim(cuda_rt, oracle_rt, shape, dim, keepdim):
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(shape).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    for m in ("sumDim", "meanDim"):
        hc = getattr(cuda_rt, m)(cx["id"], dim, keepdim)
        ho = getattr(oracle_rt, m)(ox["id"], dim, keepdim)
        red = shape[dim]
        check(cuda_rt, oracle_rt, hc, ho, rtol=1e-4, atol=1e-5 * math.sqrt(red))


@pytest.mark.parametrize("shape,dim", [([7, 9], 0), ([7, 9], 1), ([3, 5, 6], 1), ([64, 3000], -1),
                                       ([5000, 33], 0)])
def test_max_dim_values_and_indices_exact(cuda_rt, oracle_rt, shape, dim):
    rng = np.random.default_rng(5)
    x = np.round(rng.standard_normal(shape) * 4).astype(np.float32)  # many ties
    cx, ox = both(cuda_rt, oracle_rt, x)
    cv, ci = cuda_rt.maxDim(cx["id"], dim, False)
    ov, oi = oracle_rt.maxDim(ox["id"], dim, False)
    check(cuda_rt, oracle_rt, cv, ov)
    assert np.array_equal(vals(cuda_rt, ci), vals(oracle_rt, oi))


@pytest.mark.parametrize("shape", [[2, 3], [10, 10], [64, 10], [5, 1], [3, 2049], [1000, 7]])
def test_argmax_bit_exact_first_index(cuda_rt, oracle_rt, shape):
    rng = np.random.default_rng(11)
    x = np.round(rng.standard_normal(shape) * 2).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, cuda_rt.argmax(cx["id"]), oracle_rt.argmax(ox["id"]))


# rows of C % 4 == 0 up to 8192 take the 16-byte kernels (2052 / 4100: partly
# filled last float4 groups); 1030 and 9000 the scalar ones
@pytest.mark.parametrize("shape,dim", [([4, 10], -1), ([33, 300], -1), ([3, 1500], -1), ([2, 8192], -1),
                                       ([2, 9000], -1), ([3, 5, 7], 1), ([6, 4], 0), ([5, 2052], -1),
                                       ([7, 4100], -1), ([3, 1030], -1)])
def test_softmax_logsoftmax(cuda_rt, oracle_rt, shape, dim):
    rng = np.random.default_rng(13)
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    cx, ox = both(cuda_rt, oracle_rt, x)
    check(cuda_rt, oracle_rt, cuda_rt.softmax(cx["id"], dim), oracle_rt.softmax(ox["id"], dim), rtol=1e-5,
          atol=1e-7)
    if dim in (-1, len(shape) - 1):
        check(cuda_rt, oracle_rt, cuda_rt.logSoftmax(cx["id"], dim), oracle_rt.logSoftmax(ox["id"], dim),
              rtol=1e-5, atol=1e-5)


# C % 4 == 0 rows above 256 take the one-CTA-per-row 16-byte kernel (2052 / 4100:
# partly filled last float4 groups); 1030 the warp-per-row one
@pytest.mark.parametrize("B,C", [(4, 10), (64, 10), (3, 1000), (5, 2052), (3, 8192), (7, 4100), (2, 1030)])
def test_softmax_backward_family(cuda_rt, oracle_rt, B, C):
    rng = np.random.default_rng(17)
    g = rng.standard_normal((B, C)).astype(np.float32)
    s = rng.uniform(0, 1, (B, C)).astype(np.float32)
    cg, og = both(cuda_rt, oracle_rt, g)
    cs, os_ = both(cuda_rt, oracle_rt, s)
    # a row reduction (dot / sum over C) feeds every element: the reduction bar,
    # 1e-4 relative to the row's magnitude
    check(cuda_rt, oracle_rt, cuda_rt.softmaxBackward(cg["id"], cs["id"], B, C),
          oracle_rt.softmaxBackward(og["id"], os_["id"], B, C), rtol=1e-4, atol=1e-4)
    check(cuda_rt, oracle_rt, cuda_rt.logSoftmaxBackward(cg["id"], cs["id"], B, C),
          oracle_rt.logSoftmaxBackward(og["id"], os_["id"], B, C), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("B,C", [(1, 10), (64, 10), (256, 10), (7, 1000)])
@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_cross_entropy_fwd_bwd(cuda_rt, oracle_rt, B, C, reduction):
    rng = np.random.default_rng(19)
    x = (rng.standard_normal((B, C)) * 2).astype(np.float32)
    t = rng.integers(-1, C + 1, B).astype(np.float32)  # out-of-range targets are clamped
    cx, ox = both(cuda_rt, oracle_rt, x)
    ct, ot = both(cuda_rt, oracle_rt, t)
    check(cuda_rt, oracle_rt, cuda_rt.crossEntropy(cx["id"], ct["id"]), oracle_rt.crossEntropy(ox["id"], ot["id"]),
          rtol=1e-5, atol=1e-5)
    go = np.full(1 if reduction != "none" else B, 0.7, np.float32)
    cgo, ogo = both(cuda_rt, oracle_rt, go)
    check(cuda_rt, oracle_rt, cuda_rt.crossEntropyBackward(cgo["id"], cx["id"], ct["id"], reduction),
          oracle_rt.crossEntropyBackward(ogo["id"], ox["id"], ot["id"], reduction), rtol=1e-5, atol=1e-7)


def _opt_tensors(cuda_rt, oracle_rt, shapes, seed, nstate):
    rng = np.random.default_rng(seed)
    out = []
    for s in shapes:
        p = (rng.standard_normal(s) * 0.02).astype(np.float32)
        g = (rng.standard_normal(s) * 1e-3).astype(np.float32)
        st = [np.abs(rng.standard_normal(s)).astype(np.float32) * 1e-4 for _ in range(nstate)]
        row = [both(cuda_rt, oracle_rt, a) for a in [p, g] + st]
        out.append(row)
    return out


@pytest.mark.parametrize("kind", ["adamW", "adam"])
@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_adam_steps_bit_exact(cuda_rt, oracle_rt, kind, wd):
    shapes = [[64, 33], [7], [1], [1000, 70], [4]]
    rows = _opt_tensors(cuda_rt, oracle_rt, shapes, 23, 2)
    lr, b1, b2, eps = 1e-3, 0.9, 0.999, 1e-8
    for step in (1, 2, 3):
        ss = lr / (1 - b1 ** step)
        isb = 1.0 / math.sqrt(1 - b2 ** step)
        if step == 2:  # the multi-tensor entry
            getattr(cuda_rt, kind + "StepMulti")(*[[r[k][0]["id"] for r in rows] for k in range(4)],
                                                 lr, b1, b2, eps, wd, ss, isb)
            getattr(oracle_rt, kind + "StepMulti")(*[[r[k][1]["id"] for r in rows] for k in range(4)],
                                                   lr, b1, b2, eps, wd, ss, isb)
        else:
            for r in rows:
                getattr(cuda_rt, kind + "Step")(*[r[k][0]["id"] for k in range(4)], lr, b1, b2, eps, wd, ss, isb)
                getattr(oracle_rt, kind + "Step")(*[r[k][1]["id"] for k in range(4)], lr, b1, b2, eps, wd, ss, isb)
    for r in rows:
        for k in (0, 2, 3):
            check(cuda_rt, oracle_rt, r[k][0], r[k][1])


@pytest.mark.parametrize("momentum,nesterov,damp,wd", [(0.9, True, 0.0, 0.0), (0.9, False, 0.1, 5e-4),
                                                       (0.0, False, 0.0, 0.01)])
def test_sgd_steps_bit_exact(cuda_rt, oracle_rt, momentum, nesterov, damp, wd):
    rows = _opt_tensors(cuda_rt, oracle_rt, [[300, 7], [5], [4096]], 29, 1)
    for step in range(3):
        if step == 1:
            cuda_rt.sgdStepMulti(*[[r[k][0]["id"] for r in rows] for k in range(3)], 0.05, momentum, wd, damp,
                                 nesterov)
            oracle_rt.sgdStepMulti(*[[r[k][1]["id"] for r in rows] for k in range(3)], 0.05, momentum, wd, damp,
                                   nesterov)
        else:
            for r in rows:
                cuda_rt.sgdStep(*[r[k][0]["id"] for k in range(3)], 0.05, momentum, wd, damp, nesterov)
                oracle_rt.sgdStep(*[r[k][1]["id"] for k in range(3)], 0.05, momentum, wd, damp, nesterov)
    for r in rows:
        check(cuda_rt, oracle_rt, r[0][0], r[0][1])
        check(cuda_rt, oracle_rt, r[2][0], r[2][1])


def test_optimizer_length_mismatch_raises(cuda_rt):
    p = cuda_rt.zeros([4], "float32")
    g = cuda_rt.zeros([5], "float32")
    with pytest.raises(RuntimeError, match="lengths must match"):
        cuda_rt.adamWStep(p["id"], g["id"], p["id"], p["id"], 1e-3, 0.9, 0.999, 1e-8, 0.0, 1.0, 1.0)


def test_destroy_and_unknown_id(cuda_rt):
    h = cuda_rt.zeros([3], "float32")
    cuda_rt.destroy(h["id"])
    cuda_rt.destroy(h["id"])  # second destroy is a no-op, as in the reference
    with pytest.raises(RuntimeError, match="Unknown tensor id"):
        cuda_rt.toList(h["id"])


def test_kernels_actually_launch(cuda_rt):
    before = cuda_rt.kernelLaunches()
    x = cuda_rt.rand([1000], "float32")
    cuda_rt.relu(x["id"])
    assert cuda_rt.kernelLaunches() >= before + 2
