"""CudaRuntime: the reference runtime's method surface over libtpcuda.

``TorchPyodideRuntime`` (runtime/src/runtime.ts:17-1212) is what the reference
``torch`` package calls for every tensor op; ``CudaRuntime`` exposes the same
camelCase methods with the same arguments, returning the same
``{"id", "shape", "dtype"}`` dicts (runtime/src/ops/types.ts:10-15), so
``tpcuda.shim.install(CudaRuntime())`` lets the unmodified reference package
run on a B200.  Every method is one ctypes call into libtpcuda.so; errors come
back as ``TpError`` (a RuntimeError), which is what the reference's
try/except fallbacks expect.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import DTYPE_CODE, DTYPES, Handle, check, i64arr

BIN = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "maximum": 5, "minimum": 6,
       "eq": 10, "ne": 11, "lt": 12, "le": 13, "gt": 14, "ge": 15}
UN = {"neg": 0, "abs": 1, "sqrt": 2, "exp": 3, "log": 4, "relu": 5, "rsqrt": 6, "reciprocal": 7,
      "square": 8, "sigmoid": 9, "tanh": 10}


def _prod(shape) -> int:
    r = 1
    for s in shape:
        r *= int(s)
    return r


def _dtype_code(dtype: str | None) -> int:
    if dtype is None:
        return -1
    try:
        return DTYPE_CODE[str(dtype)]
    except KeyError:
        raise _lib.TpError(-1, f"Unsupported dtype: {dtype}. Supported dtypes: {', '.join(DTYPES)}.") from None


class CudaRuntime:
    """Host mirror of TorchPyodideRuntime over the CUDA backend."""

    def __init__(self, device: int = 0) -> None:
        self.lib = _lib.load()
        check(self.lib.tp_init(int(device)))
        self._h = Handle()

    # ---- helpers ----------------------------------------------------------
    def _out(self) -> dict:
        return self._h.to_dict()

    def _call(self, fn, *args) -> dict:
        check(fn(*args, ctypes.byref(self._h)))
        return self._h.to_dict()

    # ---- device / frames (runtime.ts:1025-1090) ---------------------------
    def init(self, *_a) -> None:
        return None

    def isAvailable(self) -> bool:
        return bool(self.lib.tp_is_available())

    def isInitialized(self) -> bool:
        return True

    def deviceCount(self) -> int:
        n = ctypes.c_int(0)
        check(self.lib.tp_device_count(ctypes.byref(n)))
        return int(n.value)

    def currentDevice(self) -> int:
        return 0

    def getDeviceName(self, *_a) -> str:
        buf = ctypes.create_string_buffer(256)
        check(self.lib.tp_device_name(buf, 256))
        return buf.value.decode()

    def getDeviceProperties(self, *_a) -> dict:
        return {"name": self.getDeviceName(), "backend": "cuda"}

    def memoryAllocated(self, *_a) -> int:
        v = ctypes.c_int64(0)
        check(self.lib.tp_memory_allocated(ctypes.byref(v)))
        return int(v.value)

    def memoryReserved(self, *_a) -> int:
        v = ctypes.c_int64(0)
        check(self.lib.tp_memory_reserved(ctypes.byref(v)))
        return int(v.value)

    def beginFrame(self) -> None:
        """Frames batch nothing here either: every op is already queued on one stream."""

    def endFrame(self) -> None:
        return None

    def cancelFrame(self) -> None:
        return None

    def synchronize(self) -> None:
        check(self.lib.tp_synchronize())

    def stream(self) -> int:
        p = ctypes.c_void_p()
        check(self.lib.tp_get_stream(ctypes.byref(p)))
        return int(p.value or 0)

    def kernelLaunches(self) -> int:
        v = ctypes.c_int64(0)
        check(self.lib.tp_kernel_launches(ctypes.byref(v)))
        return int(v.value)

    def devicePtr(self, tid: int) -> int:
        p = ctypes.c_void_p()
        check(self.lib.tp_device_ptr(int(tid), ctypes.byref(p)))
        return int(p.value or 0)

    # ---- creation (creationOps.ts) -----------------------------------------
    def tensorFromData(self, data, shape, dtype):
        code = _dtype_code(dtype)
        n = _prod(shape)
        if isinstance(data, np.ndarray):
            arr = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        else:
            vals = list(data)
            if dtype == "bool":
                vals = [1.0 if v else 0.0 for v in vals]
            elif dtype.startswith("uint"):
                vals = [float(max(0, math.trunc(v))) for v in vals]
            elif dtype.startswith("int"):
                vals = [float(math.trunc(v)) for v in vals]
            arr = np.asarray(vals, dtype=np.float32)
        if arr.size != n:
            raise _lib.TpError(-1, f"tensorFromData expected {n} values, got {arr.size}.")
        return self._call(self.lib.tp_tensor_from_data, arr.ctypes.data_as(ctypes.c_void_p), i64arr(shape),
                          len(shape), code)

    def full(self, shape, value, dtype):
        return self._call(self.lib.tp_full, i64arr(shape), len(shape), _dtype_code(dtype), float(value))

    def zeros(self, shape, dtype):
        return self.full(shape, 0.0, dtype)

    def ones(self, shape, dtype):
        return self.full(shape, 1.0, dtype)

    def empty(self, shape, dtype):
        return self.full(shape, 0.0, dtype)

    def fullLike(self, tid, value, dtype=None):
        return self._call(self.lib.tp_full_like, int(tid), _dtype_code(dtype), float(value))

    def zerosLike(self, tid, dtype=None):
        return self.fullLike(tid, 0.0, dtype)

    def onesLike(self, tid, dtype=None):
        return self.fullLike(tid, 1.0, dtype)

    def emptyLike(self, tid, dtype=None):
        return self.fullLike(tid, 0.0, dtype)

    def fill(self, tid, value):
        return self._call(self.lib.tp_fill, int(tid), float(value))

    def setSeed(self, seed) -> None:
        check(self.lib.tp_set_seed(int(seed) & 0xFFFFFFFF))

    def _sample(self, shape, dtype, kind, p0=0.0, p1=1.0):
        return self._call(self.lib.tp_random, i64arr(shape), len(shape), _dtype_code(dtype), kind, float(p0),
                          float(p1))

    def rand(self, shape, dtype):
        return self._sample(shape, dtype, 0)

    def randn(self, shape, dtype):
        return self._sample(shape, dtype, 1)

    def normal(self, shape, dtype, mean, std):
        return self._sample(shape, dtype, 2, mean, std)

    def bernoulli(self, shape, dtype, p):
        return self._sample(shape, dtype, 3, p)

    def exponential(self, shape, dtype, rate):
        return self._sample(shape, dtype, 4, rate)

    # ---- element-wise --------------------------------------------------------
    def _bin(self, op, a, b):
        return self._call(self.lib.tp_binary, BIN[op], int(a), int(b))

    def add(self, a, b):
        return self._bin("add", a, b)

    def sub(self, a, b):
        return self._bin("sub", a, b)

    def mul(self, a, b):
        return self._bin("mul", a, b)

    def div(self, a, b):
        return self._bin("div", a, b)

    def pow(self, a, b):
        return self._bin("pow", a, b)

    def maximum(self, a, b):
        return self._bin("maximum", a, b)

    def minimum(self, a, b):
        return self._bin("minimum", a, b)

    def eq(self, a, b):
        return self._bin("eq", a, b)

    def ne(self, a, b):
        return self._bin("ne", a, b)

    def lt(self, a, b):
        return self._bin("lt", a, b)

    def le(self, a, b):
        return self._bin("le", a, b)

    def gt(self, a, b):
        return self._bin("gt", a, b)

    def ge(self, a, b):
        return self._bin("ge", a, b)

    def mulScalar(self, tid, value):
        return self._call(self.lib.tp_mul_scalar, int(tid), float(value))

    def _un(self, op, tid):
        return self._call(self.lib.tp_unary, UN[op], int(tid))

    def relu(self, t):
        return self._un("relu", t)

    def rsqrt(self, t):
        return self._un("rsqrt", t)

    def neg(self, t):
        return self._un("neg", t)

    def abs(self, t):
        return self._un("abs", t)

    def sqrt(self, t):
        return self._un("sqrt", t)

    def exp(self, t):
        return self._un("exp", t)

    def log(self, t):
        return self._un("log", t)

    def reciprocal(self, t):
        return self._un("reciprocal", t)

    def square(self, t):
        return self._un("square", t)

    def sigmoid(self, t):
        return self._un("sigmoid", t)

    def tanh(self, t):
        return self._un("tanh", t)

    # ---- shape (shapeOps.ts) ----------------------------------------------------
    def _meta(self, tid) -> dict:
        h = Handle()
        check(self.lib.tp_meta(int(tid), ctypes.byref(h)))
        return h.to_dict()

    def reshape(self, tid, shape):
        shape = [int(s) for s in shape]
        return self._call(self.lib.tp_reshape, int(tid), i64arr(shape), len(shape))

    def flatten(self, tid, startDim=0, endDim=-1):
        shape = self._meta(tid)["shape"]
        r = len(shape)
        s = startDim + r if startDim < 0 else startDim
        e = endDim + r if endDim < 0 else endDim
        return self.reshape(tid, shape[:s] + [_prod(shape[s:e + 1])] + shape[e + 1:])

    def squeeze(self, tid, dim=None):
        shape = self._meta(tid)["shape"]
        if dim is not None:
            d = dim + len(shape) if dim < 0 else dim
            new = [s for i, s in enumerate(shape) if not (i == d and s == 1)]
        else:
            new = [s for s in shape if s != 1]
        return self.reshape(tid, new if new else [1])

    def unsqueeze(self, tid, dim):
        shape = self._meta(tid)["shape"]
        d = dim + len(shape) + 1 if dim < 0 else dim
        return self.reshape(tid, shape[:d] + [1] + shape[d:])

    def transpose2d(self, tid):
        return self.transpose(tid, 0, 1)

    def transpose(self, tid, d0, d1):
        shape = self._meta(tid)["shape"]
        r = len(shape)
        if r == 2:
            return self._call(self.lib.tp_transpose2d, int(tid))
        d0 = d0 + r if d0 < 0 else d0
        d1 = d1 + r if d1 < 0 else d1
        dims = list(range(r))
        dims[d0], dims[d1] = dims[d1], dims[d0]
        return self.permute(tid, dims)

    def permute(self, tid, dims):
        arr = (ctypes.c_int32 * max(1, len(dims)))(*[int(d) for d in dims])
        return self._call(self.lib.tp_permute, int(tid), arr, len(dims))

    def expand(self, tid, shape):
        shape = [int(s) for s in shape]
        return self._call(self.lib.tp_expand, int(tid), i64arr(shape), len(shape))

    # ---- reductions (reductionOps.ts) ---------------------------------------------
    def sum(self, tid):
        return self._call(self.lib.tp_reduce_all, int(tid), 0)

    def mean(self, tid):
        return self._call(self.lib.tp_reduce_all, int(tid), 1)

    def max(self, tid):
        return self._call(self.lib.tp_reduce_all, int(tid), 2)

    def sumDim(self, tid, dim, keepdim):
        return self._call(self.lib.tp_reduce_dim, int(tid), int(dim), 1 if keepdim else 0, 0)

    def meanDim(self, tid, dim, keepdim):
        return self._call(self.lib.tp_reduce_dim, int(tid), int(dim), 1 if keepdim else 0, 1)

    def maxDim(self, tid, dim, keepdim):
        hv, hi = Handle(), Handle()
        check(self.lib.tp_max_dim(int(tid), int(dim), 1 if keepdim else 0, ctypes.byref(hv), ctypes.byref(hi)))
        return [hv.to_dict(), hi.to_dict()]

    def argmax(self, tid):
        return self._call(self.lib.tp_argmax, int(tid))

    def softmax(self, tid, dim):
        return self._call(self.lib.tp_softmax, int(tid), int(dim))

    def logSoftmax(self, tid, dim):
        return self._call(self.lib.tp_log_softmax, int(tid), int(dim))

    def softmaxBackward(self, go, s, batchSize, numClasses):
        return self._call(self.lib.tp_softmax_backward, int(go), int(s), int(batchSize), int(numClasses))

    def logSoftmaxBackward(self, go, s, batchSize, numClasses):
        return self._call(self.lib.tp_log_softmax_backward, int(go), int(s), int(batchSize), int(numClasses))

    def crossEntropy(self, inp, tgt):
        return self._call(self.lib.tp_cross_entropy, int(inp), int(tgt))

    def crossEntropyBackward(self, go, inp, tgt, reduction):
        red = {"none": 0, "sum": 1, "mean": 2}[str(reduction)]
        return self._call(self.lib.tp_cross_entropy_backward, int(go), int(inp), int(tgt), red)

    # ---- dense contractions (arithmeticOps.ts:260-340, convOps.ts) --------------
    def matmul(self, a, b):
        return self._call(self.lib.tp_matmul, int(a), int(b))

    mm = matmul
    bmm = matmul
    mv = matmul

    def linear(self, x, weight, bias=None):
        return self._call(self.lib.tp_linear, int(x), int(weight), int(bias) if bias is not None else 0)

    def conv2d(self, inp, weight, bias, stride, padding, dilation, groups):
        if bias is not None:
            barr = np.asarray(list(bias), dtype=np.float32)
            bp, nb = barr.ctypes.data_as(_lib.F32P), int(barr.size)
        else:
            barr, bp, nb = None, None, 0
        st, pd, dl = list(stride), list(padding), list(dilation)
        return self._call(self.lib.tp_conv2d, int(inp), int(weight), bp, nb, i64arr(st), len(st), i64arr(pd),
                          len(pd), i64arr(dl), len(dl), int(groups))

    def conv2dInputBackward(self, go, weight, inputShape, gradOutputShape, stride, padding):
        st, pd = list(stride), list(padding)
        return self._call(self.lib.tp_conv2d_input_backward, int(go), int(weight), i64arr(inputShape),
                          i64arr(gradOutputShape), i64arr(st), len(st), i64arr(pd), len(pd))

    def conv2dWeightBackward(self, go, inp, weightShape, gradOutputShape, inputShape, stride, padding):
        st, pd = list(stride), list(padding)
        return self._call(self.lib.tp_conv2d_weight_backward, int(go), int(inp), i64arr(weightShape),
                          i64arr(gradOutputShape), i64arr(inputShape), i64arr(st), len(st), i64arr(pd), len(pd))

    def conv2dBiasBackward(self, go, outCh, gradOutputShape):
        return self._call(self.lib.tp_conv2d_bias_backward, int(go), int(outCh), i64arr(gradOutputShape))

    # ---- pooling (poolingOps.ts:18-48) ----------------------------------------------
    @staticmethod
    def _pool_args(kernelSize, stride, padding, dilation):
        k, s, p, d = (list(v) if v is not None else [] for v in (kernelSize, stride, padding, dilation))
        return [i64arr(k), len(k), i64arr(s), len(s), i64arr(p), len(p), i64arr(d), len(d)]

    def maxPool2d(self, inp, kernelSize, stride, padding, dilation):
        return self._call(self.lib.tp_max_pool2d, int(inp), *self._pool_args(kernelSize, stride, padding, dilation))

    def maxPool2dWithIndices(self, inp, kernelSize, stride, padding, dilation):
        hy, hi = Handle(), Handle()
        check(self.lib.tp_max_pool2d_with_indices(int(inp), *self._pool_args(kernelSize, stride, padding, dilation),
                                                  ctypes.byref(hy), ctypes.byref(hi)))
        return [hy.to_dict(), hi.to_dict()]

    def maxPool2dBackward(self, go, indices, inputShape, kernelSize, stride, padding, dilation):
        return self._call(self.lib.tp_max_pool2d_backward, int(go), int(indices), i64arr(inputShape),
                          *self._pool_args(kernelSize, stride, padding, dilation))

    # ---- normalisation (normalizationOps.ts, tensor_nn_ops.py) --------------------
    @staticmethod
    def _opt(tid):
        return int(tid) if tid is not None else 0

    def batchNorm(self, inp, weight, bias, runningMean, runningVar, eps):
        o = self._opt
        return self._call(self.lib.tp_batch_norm, int(inp), o(weight), o(bias), o(runningMean), o(runningVar),
                          float(eps))

    def batchNormTrain(self, inp, weight, bias, runningMean, runningVar, eps, momentum, fuseRelu=False):
        o = self._opt
        hs = [Handle(), Handle(), Handle()]
        check(self.lib.tp_batch_norm_train(int(inp), o(weight), o(bias), o(runningMean), o(runningVar), float(eps),
                                           float(momentum), 1 if fuseRelu else 0, *[ctypes.byref(h) for h in hs]))
        return [h.to_dict() for h in hs]

    def batchNormBackward(self, go, inp, weight, saveMean, saveInvstd, reluOut=None):
        o = self._opt
        hs = [Handle(), Handle(), Handle()]
        check(self.lib.tp_batch_norm_backward(int(go), int(inp), o(weight), int(saveMean), int(saveInvstd),
                                              o(reluOut), *[ctypes.byref(h) for h in hs]))
        return [h.to_dict() for h in hs]

    def layerNorm(self, inp, normalizedShape, gamma, beta, eps):
        h = Handle()
        check(self.lib.tp_layer_norm(int(inp), _prod(normalizedShape), self._opt(gamma), self._opt(beta),
                                     float(eps), ctypes.byref(h), None, None))
        return h.to_dict()

    def _call3(self, fn, *args):
        hs = [Handle(), Handle(), Handle()]
        check(fn(*args, *[ctypes.byref(h) for h in hs]))
        return [h.to_dict() for h in hs]

    def layerNormForward(self, inp, normalizedShape, gamma, beta, eps):
        return self._call3(self.lib.tp_layer_norm, int(inp), _prod(normalizedShape), self._opt(gamma),
                           self._opt(beta), float(eps))

    def layerNormBackward(self, go, inp, normalizedShape, gamma, saveMean, saveRstd):
        hs = self._call3(self.lib.tp_layer_norm_backward, int(go), int(inp), _prod(normalizedShape),
                         self._opt(gamma), int(saveMean), int(saveRstd))
        nshape = [int(s) for s in normalizedShape]
        for h in hs[1:]:
            h["shape"] = nshape
        return hs

    # ---- optimizer steps (in place, return None) ---------------------------------
    def adamWStep(self, p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        check(self.lib.tp_adamw_step(int(p), int(g), int(m), int(v), lr, b1, b2, eps, wd, stepSize, invSqrtBc2))

    def adamStep(self, p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        check(self.lib.tp_adam_step(int(p), int(g), int(m), int(v), lr, b1, b2, eps, wd, stepSize, invSqrtBc2))

    def sgdStep(self, p, g, buf, lr, momentum, wd, dampening, nesterov):
        check(self.lib.tp_sgd_step(int(p), int(g), int(buf), lr, momentum, wd, dampening, 1 if nesterov else 0))

    def adamWStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        check(self.lib.tp_adamw_step_multi(i64arr(ps), i64arr(gs), i64arr(ms), i64arr(vs), len(ps), lr, b1, b2, eps,
                                           wd, stepSize, invSqrtBc2))

    def adamStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        check(self.lib.tp_adam_step_multi(i64arr(ps), i64arr(gs), i64arr(ms), i64arr(vs), len(ps), lr, b1, b2, eps,
                                          wd, stepSize, invSqrtBc2))

    def sgdStepMulti(self, ps, gs, bufs, lr, momentum, wd, dampening, nesterov):
        check(self.lib.tp_sgd_step_multi(i64arr(ps), i64arr(gs), i64arr(bufs), len(ps), lr, momentum, wd, dampening,
                                         1 if nesterov else 0))

    # ---- the other fused optimizer steps (runtime.ts:683-801), in place ----------
    def rmspropStep(self, p, g, squareAvg, momentumBuf, lr, alpha, eps, weightDecay, momentum):
        check(self.lib.tp_rmsprop_step(int(p), int(g), int(squareAvg), int(momentumBuf), lr, alpha, eps, weightDecay,
                                       momentum))

    def adagradStep(self, p, g, sumSquares, lr, eps, weightDecay):
        check(self.lib.tp_adagrad_step(int(p), int(g), int(sumSquares), lr, eps, weightDecay))

    def adamaxStep(self, p, g, expAvg, expInf, lr, b1, b2, eps, wd, stepSize, biasCorrection1):
        check(self.lib.tp_adamax_step(int(p), int(g), int(expAvg), int(expInf), lr, b1, b2, eps, wd, stepSize,
                                      biasCorrection1))

    def nadamStep(self, p, g, expAvg, expAvgSq, lr, b1, b2, eps, wd, stepSize, mu):
        check(self.lib.tp_nadam_step(int(p), int(g), int(expAvg), int(expAvgSq), lr, b1, b2, eps, wd, stepSize, mu))

    def radamStep(self, p, g, expAvg, expAvgSq, lr, b1, b2, eps, wd, stepSize, beta1PowT, beta2PowT, stepCount=0):
        check(self.lib.tp_radam_step(int(p), int(g), int(expAvg), int(expAvgSq), lr, b1, b2, eps, wd, stepSize,
                                     beta1PowT, beta2PowT, int(stepCount)))

    def rmspropStepMulti(self, ps, gs, sqs, mbs, lr, alpha, eps, weightDecay, momentum):
        check(self.lib.tp_rmsprop_step_multi(i64arr(ps), i64arr(gs), i64arr(sqs), i64arr(mbs), len(ps), lr, alpha,
                                             eps, weightDecay, momentum))

    def adagradStepMulti(self, ps, gs, sums, lr, eps, weightDecay):
        check(self.lib.tp_adagrad_step_multi(i64arr(ps), i64arr(gs), i64arr(sums), len(ps), lr, eps, weightDecay))

    def adamaxStepMulti(self, ps, gs, ms, us, lr, b1, b2, eps, wd, stepSize, biasCorrection1):
        check(self.lib.tp_adamax_step_multi(i64arr(ps), i64arr(gs), i64arr(ms), i64arr(us), len(ps), lr, b1, b2, eps,
                                            wd, stepSize, biasCorrection1))

    def nadamStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, mu):
        check(self.lib.tp_nadam_step_multi(i64arr(ps), i64arr(gs), i64arr(ms), i64arr(vs), len(ps), lr, b1, b2, eps,
                                           wd, stepSize, mu))

    def radamStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, beta1PowT, beta2PowT, stepCount):
        check(self.lib.tp_radam_step_multi(i64arr(ps), i64arr(gs), i64arr(ms), i64arr(vs), len(ps), lr, b1, b2, eps,
                                           wd, stepSize, beta1PowT, beta2PowT, int(stepCount)))

    # ---- conv2d with a device bias (no readback of the bias) ---------------------
    def conv2dDevBias(self, inp, weight, bias, stride, padding, dilation, groups):
        st, pd, dl = list(stride), list(padding), list(dilation)
        return self._call(self.lib.tp_conv2d_dev_bias, int(inp), int(weight), int(bias) if bias is not None else 0,
                          i64arr(st), len(st), i64arr(pd), len(pd), i64arr(dl), len(dl), int(groups))

    # ---- bulk bytes (checkpoints) and pinned uploads ------------------------------
    def toBytes(self, tid, fmt: str = "float32") -> bytes:
        """The tensor's values as little-endian float32 (or int64) bytes."""
        code = {"float32": 0, "int64": 1}[fmt]
        n = _prod(self._meta(tid)["shape"])
        buf = ctypes.create_string_buffer(n * (4 if code == 0 else 8))
        check(self.lib.tp_to_bytes(int(tid), buf, len(buf), code))
        return buf.raw

    def fromBytes(self, data, shape, dtype, fmt: str = "float32"):
        code = {"float32": 0, "int64": 1}[fmt]
        mv = memoryview(data).cast("B")
        arr = (ctypes.c_char * len(mv)).from_buffer_copy(mv) if mv.readonly else (ctypes.c_char * len(mv)).from_buffer(mv)
        return self._call(self.lib.tp_from_bytes, arr, len(mv), code, i64arr(shape), len(shape), _dtype_code(dtype))

    def hostAlloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(self.lib.tp_host_alloc(int(nbytes), ctypes.byref(p)))
        return int(p.value or 0)

    def hostFree(self, ptr: int) -> None:
        check(self.lib.tp_host_free(ctypes.c_void_p(ptr)))

    def tensorFromHostAsync(self, host_ptr: int, shape, dtype="float32", defer: bool = False):
        """Upload from pinned host memory on the copy stream; returns (handle,
        ticket).  defer: later kernels wait only after ticketUse(ticket)."""
        h, t = Handle(), ctypes.c_int64(0)
        check(self.lib.tp_tensor_from_host_async(ctypes.c_void_p(host_ptr), i64arr(shape), len(shape),
                                                 _dtype_code(dtype), 1 if defer else 0, ctypes.byref(h),
                                                 ctypes.byref(t)))
        return h.to_dict(), int(t.value)

    def ticketUse(self, ticket: int) -> None:
        check(self.lib.tp_ticket_use(int(ticket)))

    def gatherRows(self, tid, rows):
        """src[rows] along dim 0 as a new tensor (a DataLoader batch)."""
        rows = [int(r) for r in rows]
        return self._call(self.lib.tp_gather_rows, int(tid), i64arr(rows), len(rows))

    def ticketWait(self, ticket: int) -> None:
        check(self.lib.tp_ticket_wait(int(ticket)))

    # ---- readback / lifetime (runtime.ts:1046-1054) -------------------------------
    def toNumpy(self, tid) -> np.ndarray:
        meta = self._meta(tid)
        n = _prod(meta["shape"])
        out = np.empty(n, np.float32)
        check(self.lib.tp_to_host(int(tid), out.ctypes.data_as(ctypes.c_void_p), n))
        return out

    def toList(self, tid):
        meta = self._meta(tid)
        vals = self.toNumpy(tid).tolist()
        dt = meta["dtype"]
        if dt == "bool":
            return [1 if v != 0 else 0 for v in vals]
        if dt.startswith("int") or dt.startswith("uint"):
            return [int(math.trunc(v)) for v in vals]
        return vals

    def destroy(self, tid) -> None:
        check(self.lib.tp_destroy(int(tid)))
