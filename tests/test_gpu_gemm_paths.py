"""The contraction engines (tcgen05 3xTF32 tensor-core kernel with TMA-fed or
gathered operand tiles, CUDA-core fp32 kernel) against the oracle, plus the
tensor-core kernel's status word."""
import ctypes

import numpy as np
import pytest

from test_gpu_dense import close_scaled
from test_gpu_ops import both

pytestmark = pytest.mark.gpu


def status(rt):
    v = ctypes.c_int(0)
    assert rt.lib.tp_gemm_status(ctypes.byref(v), 1) == 0
    return v.value


@pytest.fixture(params=[0, 1, 2, 3, 4],
                ids=["tcgen05_tma", "cuda_cores", "tcgen05_gather", "tcgen05_tma_single", "tcgen05_tma_pairs"])
def path(request, cuda_rt):
    assert cuda_rt.lib.tp_set_gemm_path(request.param) == 0
    yield request.param
    cuda_rt.lib.tp_set_gemm_path(0)


@pytest.mark.parametrize("M,K,N", [(128, 32, 128), (200, 70, 50), (64, 1000, 16), (512, 4096, 384),
                                   (1000, 33, 300)])
def test_matmul_paths(cuda_rt, oracle_rt, path, M, K, N):
    rng = np.random.default_rng(M + K + N)
    ca, oa = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (M, K)))
    cb, ob = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (K, N)))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.matmul(ca["id"], cb["id"]), oracle_rt.matmul(oa["id"], ob["id"]))
    assert status(cuda_rt) == 0


def test_matmul_long_k_accuracy(cuda_rt, oracle_rt):
    """K = 8192 (the largest matmul config): 3xTF32 must hold fp32 accuracy."""
    rng = np.random.default_rng(1)
    M, K, N = 256, 8192, 256
    ca, oa = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (M, K)))
    cb, ob = both(cuda_rt, oracle_rt, rng.uniform(-1, 1, (K, N)))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.matmul(ca["id"], cb["id"]), oracle_rt.matmul(oa["id"], ob["id"]),
                 rel=2e-5)
    assert status(cuda_rt) == 0


@pytest.mark.parametrize("xs,ws", [([8, 64, 16, 16], [128, 64, 3, 3]), ([4, 3, 32, 32], [64, 3, 3, 3]),
                                   ([16, 256, 4, 4], [512, 256, 3, 3]), ([2, 64, 20, 20], [64, 64, 3, 3]),
                                   ([2, 32, 9, 9], [64, 32, 5, 5])])
def test_conv_paths(cuda_rt, oracle_rt, path, xs, ws):
    rng = np.random.default_rng(sum(xs))
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(xs))
    cw, ow = both(cuda_rt, oracle_rt, rng.standard_normal(ws) * 0.1)
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2d(cx["id"], cw["id"], None, [1], [1], [1], 1),
                 oracle_rt.conv2d(ox["id"], ow["id"], None, [1], [1], [1], 1))
    y = oracle_rt.conv2d(ox["id"], ow["id"], None, [1], [1], [1], 1)
    cg, og = both(cuda_rt, oracle_rt, rng.standard_normal(y["shape"]))
    ys = y["shape"]
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dInputBackward(cg["id"], cw["id"], xs, ys, [1], [1]),
                 oracle_rt.conv2dInputBackward(og["id"], ow["id"], xs, ys, [1], [1]))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dWeightBackward(cg["id"], cx["id"], ws, ys, xs, [1], [1]),
                 oracle_rt.conv2dWeightBackward(og["id"], ox["id"], ws, ys, xs, [1], [1]))
    assert status(cuda_rt) == 0


# every convolution shape of the VGG-11-BN step at per-rank batch 16 (the 8-GPU
# split of a 128 batch) and 4
VGG_SHAPES = [(3, 64, 32), (64, 128, 16), (128, 256, 8), (256, 256, 8), (256, 512, 4), (512, 512, 4),
              (512, 512, 2)]


@pytest.mark.parametrize("cin,cout,hw", VGG_SHAPES)
@pytest.mark.parametrize("batch", [4, 16])
def test_vgg_conv_shapes(cuda_rt, oracle_rt, path, cin, cout, hw, batch):
    xs, ws = [batch, cin, hw, hw], [cout, cin, 3, 3]
    rng = np.random.default_rng(cin * 7 + cout + hw + batch)
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(xs))
    cw, ow = both(cuda_rt, oracle_rt, rng.standard_normal(ws) * 0.05)
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2d(cx["id"], cw["id"], None, [1], [1], [1], 1),
                 oracle_rt.conv2d(ox["id"], ow["id"], None, [1], [1], [1], 1))
    ys = [batch, cout, hw, hw]
    cg, og = both(cuda_rt, oracle_rt, rng.standard_normal(ys))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dInputBackward(cg["id"], cw["id"], xs, ys, [1], [1]),
                 oracle_rt.conv2dInputBackward(og["id"], ow["id"], xs, ys, [1], [1]))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dWeightBackward(cg["id"], cx["id"], ws, ys, xs, [1], [1]),
                 oracle_rt.conv2dWeightBackward(og["id"], ox["id"], ws, ys, xs, [1], [1]))
    assert status(cuda_rt) == 0


@pytest.mark.parametrize("xs,ws,st,pd", [([2, 3, 20, 20], [16, 3, 7, 7], 2, 3), ([3, 2, 11, 13], [8, 2, 3, 3], 2, 1),
                                         ([2, 4, 9, 9], [12, 4, 5, 5], 3, 2),
                                         # the network stem at a small batch: all three passes take the
                                         # space-to-depth route onto the TMA kernels on the default engine
                                         ([2, 3, 64, 64], [64, 3, 7, 7], 2, 3), ([1, 3, 37, 30], [32, 3, 5, 5], 2, 2)])
def test_conv_strided_few_channels(cuda_rt, oracle_rt, path, xs, ws, st, pd):
    """Strided convolutions with few input channels (a network stem): forward,
    data gradient and weight gradient against the oracle (stride 2 on the
    default engine: space-to-depth onto the TMA kernels; other strides: the
    phase-decomposed CUDA-core data gradient and the gather kernels)."""
    rng = np.random.default_rng(sum(xs) + st)
    cx, ox = both(cuda_rt, oracle_rt, rng.standard_normal(xs))
    cw, ow = both(cuda_rt, oracle_rt, rng.standard_normal(ws) * 0.1)
    y = oracle_rt.conv2d(ox["id"], ow["id"], None, [st], [pd], [1], 1)
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2d(cx["id"], cw["id"], None, [st], [pd], [1], 1), y)
    ys = y["shape"]
    cg, og = both(cuda_rt, oracle_rt, rng.standard_normal(ys))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dInputBackward(cg["id"], cw["id"], xs, ys, [st], [pd]),
                 oracle_rt.conv2dInputBackward(og["id"], ow["id"], xs, ys, [st], [pd]))
    close_scaled(cuda_rt, oracle_rt, cuda_rt.conv2dWeightBackward(cg["id"], cx["id"], ws, ys, xs, [st], [pd]),
                 oracle_rt.conv2dWeightBackward(og["id"], ox["id"], ws, ys, xs, [st], [pd]))
    assert status(cuda_rt) == 0
