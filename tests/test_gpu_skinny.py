"""Products with a side of at most 16 rows (the 512 -> 10 classifier of a CNN
and its gradients) run on the skinny CUDA-core kernel; checked against a
float64 product of the same operands for every operand layout, with and
without a k split and a bias."""
import ctypes

import numpy as np
import pytest

from test_gpu_tma import dev, empty, free, read, status  # noqa: F401

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(10, 512, 1024), (1024, 10, 512), (3, 700, 300), (700, 1, 64), (16, 16, 4096),
                                   (5, 2000, 40), (128, 10, 784)])
@pytest.mark.parametrize("a_t", [0, 1])
@pytest.mark.parametrize("b_t", [0, 1])
def test_skinny_gemm(cuda_rt, M, N, K, a_t, b_t):
    rt = cuda_rt
    rng = np.random.default_rng(M + 3 * N + 7 * K + a_t + 2 * b_t)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    pa, pb, pbias, pc = dev(rt, A.T if a_t else A), dev(rt, B.T if b_t else B), dev(rt, bias), empty(rt, M * N)
    assert rt.lib.tpk_gemm(ctypes.c_void_p(pa), a_t, ctypes.c_void_p(pb), b_t, ctypes.c_void_p(pc), M, N, K,
                           ctypes.c_void_p(pbias)) == 0
    got = read(rt, pc, (M, N)).astype(np.float64)
    assert status(rt) == 0
    free(rt, pa, pb, pbias, pc)
    ref = A.astype(np.float64) @ B.astype(np.float64) + bias
    scale = max(1e-30, float(np.max(np.abs(ref))))
    assert float(np.max(np.abs(got - ref))) <= 1e-5 * scale
