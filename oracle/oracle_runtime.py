"""CPU oracle runtime: the reference runtime's op surface over oracle/liboracle.so.

TEST INFRASTRUCTURE ONLY.  ``OracleRuntime`` restates, on the host, the method
surface of ``TorchPyodideRuntime`` (runtime/src/runtime.ts:17-1212) for the hot
path, with the per-invocation arithmetic of each WGSL entry point done by the C
functions in oracle/oracle.c.  It exists to check the CUDA backend: tests,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm use it;
the CUDA product path (``tpcuda``) never imports it.

Conventions copied from the reference runtime (they define what a caller sees):
  * every tensor is stored as float32 whatever its dtype tag
    (runtime/src/ops/device.ts:362-364, creationOps.ts:31-33);
  * ops return ``{"id", "shape", "dtype"}`` (runtime/src/ops/types.ts:10-15),
    fresh buffers every time, except the optimizer steps which update
    param / state in place and return None;
  * ``toList`` decodes integer and bool dtypes with trunc / !=0
    (runtime/src/ops/device.ts:38-54);
  * the seed counter starts at 42 and is bumped by every sampling call
    (creationOps.ts:17,81).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)
I32P = ctypes.POINTER(ctypes.c_int32)
I64P = ctypes.POINTER(ctypes.c_int64)


class ConvParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in
                ("N", "Cin", "Cout", "H", "W", "OH", "OW", "KH", "KW", "SH", "SW", "PH", "PW", "groups")]


class PoolParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in
                ("N", "C", "H", "W", "OH", "OW", "KH", "KW", "SH", "SW", "PH", "PW", "DH", "DW")]


def build_oracle() -> str:
    """Compile liboracle.so with oracle/Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    """The loaded oracle library (built on first use if it is missing)."""
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "oracle.c")
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
            build_oracle()
        L = ctypes.CDLL(_LIB_PATH)
        L.or_fill.argtypes = [F32P, ctypes.c_int64, ctypes.c_float]
        L.or_random.argtypes = [F32P, ctypes.c_int64, ctypes.c_uint32, ctypes.c_int, ctypes.c_float, ctypes.c_float]
        L.or_binary_bcast.argtypes = [ctypes.c_int, F32P, I64P, F32P, I64P, F32P, I64P, ctypes.c_int]
        L.or_unary.argtypes = [ctypes.c_int, F32P, F32P, ctypes.c_int64]
        L.or_mul_scalar.argtypes = [F32P, ctypes.c_float, F32P, ctypes.c_int64]
        L.or_transpose2d.argtypes = [F32P, F32P, ctypes.c_int64, ctypes.c_int64]
        L.or_permute.argtypes = [F32P, I64P, ctypes.POINTER(ctypes.c_int), ctypes.c_int, F32P]
        L.or_expand.argtypes = [F32P, I64P, F32P, I64P, ctypes.c_int]
        L.or_matmul.argtypes = [F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int]
        L.or_reduce_all.argtypes = [F32P, ctypes.c_int64, ctypes.c_int]
        L.or_reduce_all.restype = ctypes.c_float
        L.or_reduce_dim.argtypes = [F32P, F32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        L.or_argmax.argtypes = [F32P, I32P, ctypes.c_int64, ctypes.c_int64]
        L.or_max_dim.argtypes = [F32P, F32P, I32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.or_softmax.argtypes = [F32P, F32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.or_log_softmax.argtypes = [F32P, F32P, ctypes.c_int64, ctypes.c_int64]
        L.or_softmax_backward.argtypes = [F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64]
        L.or_log_softmax_backward.argtypes = [F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64]
        L.or_cross_entropy.argtypes = [F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64]
        L.or_cross_entropy_backward.argtypes = [F32P, ctypes.c_int, F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_float]
        CP = ctypes.POINTER(ConvParams)
        L.or_conv2d.argtypes = [F32P, F32P, F32P, F32P, CP]
        L.or_conv2d_input_backward.argtypes = [F32P, F32P, F32P, CP]
        L.or_conv2d_weight_backward.argtypes = [F32P, F32P, F32P, CP]
        L.or_conv2d_bias_backward.argtypes = [F32P, F32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64]
        PP = ctypes.POINTER(PoolParams)
        L.or_max_pool2d.argtypes = [F32P, F32P, I32P, PP]
        L.or_max_pool2d_backward.argtypes = [F32P, I32P, F32P, PP]
        L.or_batchnorm_eval.argtypes = [F32P, F32P, F32P, F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_float]
        L.or_batchnorm_train.argtypes = [F32P, F32P, F32P, F32P, F32P, F32P, F32P, F32P, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_float]
        L.or_batchnorm_backward.argtypes = [F32P, F32P, F32P, F32P, F32P, F32P, F32P, F32P, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64]
        L.or_layernorm.argtypes = [F32P, F32P, F32P, F32P, F32P, F32P, ctypes.c_int64, ctypes.c_int64, ctypes.c_float]
        L.or_layernorm_backward.argtypes = [F32P, F32P, F32P, F32P, F32P, F32P, F32P, F32P, ctypes.c_int64,
                                            ctypes.c_int64]
        for nm in ("or_adamw_step", "or_adam_step"):
            getattr(L, nm).argtypes = [F32P, F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 7
        L.or_sgd_step.argtypes = [F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 4 + [ctypes.c_int]
        L.or_rmsprop_step.argtypes = [F32P, F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 5
        L.or_adagrad_step.argtypes = [F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 3
        for nm in ("or_adamax_step", "or_nadam_step"):
            getattr(L, nm).argtypes = [F32P, F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 7
        L.or_radam_step.argtypes = [F32P, F32P, F32P, F32P, ctypes.c_int64] + [ctypes.c_float] * 8 + [ctypes.c_int64]
        _lib = L
    return _lib


def fp(a: np.ndarray | None):
    """float32 pointer into a C-contiguous numpy array (or NULL)."""
    if a is None:
        return ctypes.cast(None, F32P)
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(F32P)


def ip(a: np.ndarray | None):
    if a is None:
        return ctypes.cast(None, I32P)
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(I32P)


def i64arr(vals: Sequence[int]):
    arr = (ctypes.c_int64 * max(1, len(vals)))(*[int(v) for v in vals])
    return arr


# --------------------------------------------------------------------------
# Array-level helpers (used directly by the GPU parity tests as the checker).

BINOP = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "maximum": 5, "minimum": 6,
         "eq": 10, "ne": 11, "lt": 12, "le": 13, "gt": 14, "ge": 15}
UNOP = {"neg": 0, "abs": 1, "sqrt": 2, "exp": 3, "log": 4, "relu": 5, "rsqrt": 6, "reciprocal": 7,
        "square": 8, "sigmoid": 9, "tanh": 10}


def broadcast_shapes(a: Sequence[int], b: Sequence[int]) -> list[int]:
    """Right-aligned broadcast (runtime/src/ops/broadcastOps.ts:70-82)."""
    n = max(len(a), len(b))
    out = []
    for i in range(n):
        ad = a[len(a) - n + i] if len(a) - n + i >= 0 else 1
        bd = b[len(b) - n + i] if len(b) - n + i >= 0 else 1
        if ad != bd and ad != 1 and bd != 1:
            raise RuntimeError(f"Shapes [{list(a)}] and [{list(b)}] cannot be broadcast together.")
        out.append(max(ad, bd))
    return out


def binary(op: str, a: np.ndarray, a_shape, b: np.ndarray, b_shape):
    out_shape = broadcast_shapes(a_shape, b_shape)
    nd = len(out_shape)
    pa = [1] * (nd - len(a_shape)) + list(a_shape)
    pb = [1] * (nd - len(b_shape)) + list(b_shape)
    out = np.empty(int(np.prod(out_shape)) if out_shape else 1, np.float32)
    lib().or_binary_bcast(BINOP[op], fp(a), i64arr(pa), fp(b), i64arr(pb), fp(out), i64arr(out_shape), nd)
    return out, out_shape


def unary(op: str, x: np.ndarray):
    out = np.empty_like(x)
    lib().or_unary(UNOP[op], fp(x), fp(out), x.size)
    return out


def random(n: int, seed: int, kind: int = 0, p0: float = 0.0, p1: float = 1.0):
    out = np.empty(n, np.float32)
    lib().or_random(fp(out), n, seed & 0xFFFFFFFF, kind, p0, p1)
    return out


def matmul2d(A: np.ndarray, B: np.ndarray, M: int, K: int, N: int):
    C = np.empty(M * N, np.float32)
    lib().or_matmul(fp(A), fp(B), fp(C), 1, M, K, N, 0)
    return C


def conv_params(x_shape, w_shape, stride, padding) -> ConvParams:
    N, Cin, H, W = x_shape
    Cout, _, KH, KW = w_shape
    SH = stride[0] if len(stride) > 0 else 1
    SW = stride[1] if len(stride) > 1 else SH
    PH = padding[0] if len(padding) > 0 else 0
    PW = padding[1] if len(padding) > 1 else PH
    OH = (H + 2 * PH - KH) // SH + 1
    OW = (W + 2 * PW - KW) // SW + 1
    return ConvParams(N, Cin, Cout, H, W, OH, OW, KH, KW, SH, SW, PH, PW, 1)


def pool_params(x_shape, k, s, p, d) -> PoolParams:
    N, C, H, W = x_shape
    KH = k[0]
    KW = k[1] if len(k) > 1 else k[0]
    SH = s[0] if len(s) > 0 else KH
    SW = s[1] if len(s) > 1 else (s[0] if len(s) > 0 else KW)
    PH = p[0] if len(p) > 0 else 0
    PW = p[1] if len(p) > 1 else PH
    DH = d[0] if len(d) > 0 else 1
    DW = d[1] if len(d) > 1 else DH
    OH = (H + 2 * PH - (DH * (KH - 1) + 1)) // SH + 1
    OW = (W + 2 * PW - (DW * (KW - 1) + 1)) // SW + 1
    return PoolParams(N, C, H, W, OH, OW, KH, KW, SH, SW, PH, PW, DH, DW)


def _prod(shape) -> int:
    r = 1
    for s in shape:
        r *= int(s)
    return r


class OracleRuntime:
    """Host restatement of the reference runtime's hot-path method surface."""

    def __init__(self) -> None:
        lib()
        self._t: dict[int, tuple[np.ndarray, list[int], str]] = {}
        self._next = 1
        self._seed = 42

    # ---- registry -------------------------------------------------------
    def _reg(self, arr: np.ndarray, shape, dtype: str) -> dict:
        tid = self._next
        self._next += 1
        arr = np.ascontiguousarray(arr, dtype=np.float32).reshape(-1)
        self._t[tid] = (arr, [int(s) for s in shape], dtype)
        return {"id": tid, "shape": [int(s) for s in shape], "dtype": dtype}

    def _get(self, tid: int):
        try:
            return self._t[int(tid)]
        except KeyError:
            raise RuntimeError(f"Unknown tensor id: {tid}.") from None

    def array(self, tid: int) -> np.ndarray:
        return self._get(tid)[0]

    # ---- device / frames ------------------------------------------------
    def init(self, *_a):
        return None

    def isAvailable(self) -> bool:
        return True

    def isInitialized(self) -> bool:
        return True

    def deviceCount(self) -> int:
        return 1

    def currentDevice(self) -> int:
        return 0

    def getDeviceName(self, *_a) -> str:
        return "oracle-cpu"

    def getDeviceProperties(self, *_a) -> dict:
        return {"name": "oracle-cpu"}

    def memoryAllocated(self, *_a) -> int:
        return int(sum(a.nbytes for a, _, _ in self._t.values()))

    def memoryReserved(self, *_a) -> int:
        return self.memoryAllocated()

    def beginFrame(self) -> None:
        return None

    def endFrame(self) -> None:
        return None

    def cancelFrame(self) -> None:
        return None

    # ---- creation (creationOps.ts) ---------------------------------------
    def tensorFromData(self, data, shape, dtype):
        n = _prod(shape)
        if isinstance(data, np.ndarray):  # the same coercions as the list path, array-wide
            if data.size != n:
                raise RuntimeError(f"tensorFromData expected {n} values, got {data.size}.")
            a = np.asarray(data).reshape(-1)
            if dtype == "bool":
                a = (a != 0)
            elif dtype.startswith("uint"):
                a = np.maximum(np.trunc(a.astype(np.float64)), 0)
            elif dtype.startswith("int"):
                a = np.trunc(a.astype(np.float64))
            return self._reg(np.array(a, dtype=np.float32), shape, dtype)
        vals = list(data)
        if len(vals) != n:
            raise RuntimeError(f"tensorFromData expected {n} values, got {len(vals)}.")
        if dtype == "bool":
            vals = [1.0 if v else 0.0 for v in vals]
        elif dtype.startswith("int") or dtype.startswith("uint"):
            vals = [float(math.trunc(v)) if not dtype.startswith("uint") else float(max(0, math.trunc(v)))
                    for v in vals]
        return self._reg(np.array(vals, dtype=np.float32), shape, dtype)

    def _coerce(self, value: float, dtype: str) -> float:
        if dtype == "bool":
            return 1.0 if value else 0.0
        if dtype.startswith("int"):
            return float(math.trunc(value))
        if dtype.startswith("uint"):
            return float(max(0, math.trunc(value)))
        return float(value)

    def full(self, shape, value, dtype):
        out = np.empty(_prod(shape), np.float32)
        lib().or_fill(fp(out), out.size, self._coerce(value, dtype))
        return self._reg(out, shape, dtype)

    def zeros(self, shape, dtype):
        return self.full(shape, 0.0, dtype)

    def ones(self, shape, dtype):
        return self.full(shape, 1.0, dtype)

    def empty(self, shape, dtype):
        return self.full(shape, 0.0, dtype)

    def fullLike(self, tid, value, dtype=None):
        _, shape, dt = self._get(tid)
        return self.full(shape, value, dtype or dt)

    def zerosLike(self, tid, dtype=None):
        return self.fullLike(tid, 0.0, dtype)

    def onesLike(self, tid, dtype=None):
        return self.fullLike(tid, 1.0, dtype)

    def emptyLike(self, tid, dtype=None):
        return self.fullLike(tid, 0.0, dtype)

    def fill(self, tid, value):
        """unaryOps.ts:171-179: a new tensor of the same shape and dtype."""
        _, shape, dt = self._get(tid)
        out = np.full(_prod(shape), np.float32(value), np.float32)
        return self._reg(out, shape, dt)

    def setSeed(self, seed) -> None:
        self._seed = int(seed)

    def _sample(self, shape, dtype, kind, p0=0.0, p1=1.0):
        seed = self._seed
        self._seed += 1
        return self._reg(random(_prod(shape), seed, kind, p0, p1), shape, dtype)

    def rand(self, shape, dtype):
        return self._sample(shape, dtype, 0)

    def randn(self, shape, dtype):
        return self._sample(shape, dtype, 1)

    def normal(self, shape, dtype, mean, std):
        return self._sample(shape, dtype, 2, mean, std)

    # ---- element-wise ----------------------------------------------------
    def _bin(self, op, a, b, out_dtype=None):
        xa, sa, da = self._get(a)
        xb, sb, _ = self._get(b)
        out, shape = binary(op, xa, sa, xb, sb)
        return self._reg(out, shape, out_dtype or da)

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
        return self._bin("eq", a, b, "bool")

    def ne(self, a, b):
        return self._bin("ne", a, b, "bool")

    def lt(self, a, b):
        return self._bin("lt", a, b, "bool")

    def le(self, a, b):
        return self._bin("le", a, b, "bool")

    def gt(self, a, b):
        return self._bin("gt", a, b, "bool")

    def ge(self, a, b):
        return self._bin("ge", a, b, "bool")

    def mulScalar(self, tid, value):
        x, shape, dt = self._get(tid)
        out = np.empty_like(x)
        lib().or_mul_scalar(fp(x), float(value), fp(out), x.size)
        return self._reg(out, shape, dt)

    def _un(self, op, tid):
        x, shape, dt = self._get(tid)
        return self._reg(unary(op, x), shape, dt)

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

    # ---- shape (shapeOps.ts) --------------------------------------------
    def reshape(self, tid, shape):
        x, _, dt = self._get(tid)
        shape = [int(s) for s in shape]
        if _prod(shape) != x.size:
            raise RuntimeError(f"reshape: product {shape} != {x.size}")
        return self._reg(x.copy(), shape, dt)

    def flatten(self, tid, startDim=0, endDim=-1):
        _, shape, _ = self._get(tid)
        r = len(shape)
        s = startDim + r if startDim < 0 else startDim
        e = endDim + r if endDim < 0 else endDim
        new = shape[:s] + [_prod(shape[s:e + 1])] + shape[e + 1:]
        return self.reshape(tid, new)

    def squeeze(self, tid, dim=None):
        _, shape, _ = self._get(tid)
        if dim is not None:
            d = dim + len(shape) if dim < 0 else dim
            new = [s for i, s in enumerate(shape) if not (i == d and s == 1)]
        else:
            new = [s for s in shape if s != 1]
        return self.reshape(tid, new if new else [1])

    def unsqueeze(self, tid, dim):
        _, shape, _ = self._get(tid)
        d = dim + len(shape) + 1 if dim < 0 else dim
        return self.reshape(tid, shape[:d] + [1] + shape[d:])

    def transpose2d(self, tid):
        return self.transpose(tid, 0, 1)

    def transpose(self, tid, d0, d1):
        x, shape, dt = self._get(tid)
        r = len(shape)
        d0 = d0 + r if d0 < 0 else d0
        d1 = d1 + r if d1 < 0 else d1
        if r == 2:
            out = np.empty_like(x)
            lib().or_transpose2d(fp(x), fp(out), shape[0], shape[1])
            return self._reg(out, [shape[1], shape[0]], dt)
        dims = list(range(r))
        dims[d0], dims[d1] = dims[d1], dims[d0]
        return self.permute(tid, dims)

    def permute(self, tid, dims):
        x, shape, dt = self._get(tid)
        if len(dims) != len(shape):
            raise RuntimeError("permute: dims length mismatch")
        out = np.empty_like(x)
        cd = (ctypes.c_int * len(dims))(*[int(d) for d in dims])
        lib().or_permute(fp(x), i64arr(shape), cd, len(shape), fp(out))
        return self._reg(out, [shape[d] for d in dims], dt)

    def expand(self, tid, shape):
        x, sx, dt = self._get(tid)
        shape = [int(s) for s in shape]
        padded = [1] * (len(shape) - len(sx)) + sx
        out = np.empty(_prod(shape), np.float32)
        lib().or_expand(fp(x), i64arr(padded), fp(out), i64arr(shape), len(shape))
        return self._reg(out, shape, dt)

    # ---- matmul (arithmeticOps.ts:260-340) -------------------------------
    def matmul(self, a, b):
        xa, sa, da = self._get(a)
        xb, sb, db = self._get(b)
        if len(sa) == 2 and len(sb) == 1:
            m, k = sa
            if k != sb[0]:
                raise RuntimeError(f"matmul dimension mismatch: [{m},{k}] x [{sb[0]}].")
            out = matmul2d(xa, xb, m, k, 1)
            return self._reg(out, [m, 1], da)
        if len(sa) == 1 and len(sb) == 2:
            k, n = sa[0], sb[1]
            if k != sb[0]:
                raise RuntimeError(f"matmul dimension mismatch: [{k}] x [{sb[0]},{n}].")
            return self._reg(matmul2d(xa, xb, 1, k, n), [1, n], db)
        if len(sa) == 3 and len(sb) == 3:
            bt, m, k = sa
            if bt != sb[0] or k != sb[1]:
                raise RuntimeError("matmul dimension mismatch")
            n = sb[2]
            out = np.empty(bt * m * n, np.float32)
            lib().or_matmul(fp(xa), fp(xb), fp(out), bt, m, k, n, 1)
            return self._reg(out, [bt, m, n], da)
        if len(sa) == 2 and len(sb) == 2:
            m, k = sa
            if k != sb[0]:
                raise RuntimeError(f"matmul dimension mismatch: [{m},{k}] x [{sb[0]},{sb[1]}].")
            return self._reg(matmul2d(xa, xb, m, k, sb[1]), [m, sb[1]], da)
        if len(sa) >= 3 and len(sb) == 2:
            bt = _prod(sa[:-2])
            m, k = sa[-2:]
            n = sb[1]
            if k != sb[0]:
                raise RuntimeError("matmul dimension mismatch")
            out = np.empty(bt * m * n, np.float32)
            lib().or_matmul(fp(xa), fp(xb), fp(out), bt, m, k, n, 0)
            return self._reg(out, [bt, m, n], da)
        raise RuntimeError(f"matmul unsupported shapes: [{sa}] and [{sb}].")

    mm = matmul
    bmm = matmul
    mv = matmul

    # ---- reductions (reductionOps.ts) ------------------------------------
    def sum(self, tid):
        x, _, dt = self._get(tid)
        return self._reg(np.array([lib().or_reduce_all(fp(x), x.size, 0)], np.float32), [], dt)

    def mean(self, tid):
        x, _, dt = self._get(tid)
        return self._reg(np.array([lib().or_reduce_all(fp(x), x.size, 1)], np.float32), [], dt)

    def max(self, tid):
        x, _, dt = self._get(tid)
        return self._reg(np.array([lib().or_reduce_all(fp(x), x.size, 2)], np.float32), [], dt)

    def _rdim(self, tid, dim, keepdim, op):
        x, shape, dt = self._get(tid)
        r = len(shape)
        d = dim + r if dim < 0 else dim
        if d < 0 or d >= r:
            raise RuntimeError(f"dim {dim} out of range for rank {r}")
        outer, red, inner = _prod(shape[:d]), shape[d], _prod(shape[d + 1:])
        out = np.empty(outer * inner, np.float32)
        lib().or_reduce_dim(fp(x), fp(out), outer, red, inner, op)
        new = [1 if i == d else s for i, s in enumerate(shape)] if keepdim else [s for i, s in enumerate(shape)
                                                                                  if i != d]
        return self._reg(out, new, dt)

    def sumDim(self, tid, dim, keepdim):
        return self._rdim(tid, dim, keepdim, 0)

    def meanDim(self, tid, dim, keepdim):
        return self._rdim(tid, dim, keepdim, 1)

    def maxDim(self, tid, dim, keepdim):
        """New entry: max values and first-max indices along `dim`."""
        x, shape, dt = self._get(tid)
        r = len(shape)
        d = dim + r if dim < 0 else dim
        outer, red, inner = _prod(shape[:d]), shape[d], _prod(shape[d + 1:])
        vals = np.empty(outer * inner, np.float32)
        idx = np.empty(outer * inner, np.int32)
        lib().or_max_dim(fp(x), fp(vals), ip(idx), outer, red, inner)
        new = [1 if i == d else s for i, s in enumerate(shape)] if keepdim else [s for i, s in enumerate(shape)
                                                                                  if i != d]
        return [self._reg(vals, new, dt), self._reg(idx.astype(np.float32), new, "int64")]

    def argmax(self, tid):
        x, shape, _ = self._get(tid)
        rows = _prod(shape[:-1])
        out = np.empty(rows, np.int32)
        lib().or_argmax(fp(x), ip(out), rows, shape[-1])
        return self._reg(out.astype(np.float32), shape[:-1] if len(shape) > 1 else [1], "int32")

    def argmin(self, tid):
        """argmin.wgsl (reductionOps.ts:140-160): first index of the minimum over
        the last dim (used only to run the reference's argmax/argmin example)."""
        x, shape, _ = self._get(tid)
        rows = _prod(shape[:-1])
        out = np.argmin(x.reshape(rows, shape[-1]), axis=1).astype(np.float32)
        return self._reg(out, shape[:-1] if len(shape) > 1 else [1], "int32")

    def softmax(self, tid, dim):
        x, shape, dt = self._get(tid)
        d = dim + len(shape) if dim < 0 else dim
        outer, axis, inner = _prod(shape[:d]), shape[d], _prod(shape[d + 1:])
        out = np.empty_like(x)
        lib().or_softmax(fp(x), fp(out), outer * inner, axis, inner)
        return self._reg(out, shape, dt)

    def logSoftmax(self, tid, dim):
        x, shape, dt = self._get(tid)
        d = dim + len(shape) if dim < 0 else dim
        outer, axis, inner = _prod(shape[:d]), shape[d], _prod(shape[d + 1:])
        out = np.empty_like(x)
        lib().or_log_softmax(fp(x), fp(out), outer * inner, axis)
        return self._reg(out, shape, dt)

    def softmaxBackward(self, go, s, batchSize, numClasses):
        g, _, dt = self._get(go)
        sv = self.array(s)
        out = np.empty(batchSize * numClasses, np.float32)
        lib().or_softmax_backward(fp(g), fp(sv), fp(out), batchSize, numClasses)
        return self._reg(out, [batchSize, numClasses], dt)

    def logSoftmaxBackward(self, go, s, batchSize, numClasses):
        g, _, dt = self._get(go)
        sv = self.array(s)
        out = np.empty(batchSize * numClasses, np.float32)
        lib().or_log_softmax_backward(fp(g), fp(sv), fp(out), batchSize, numClasses)
        return self._reg(out, [batchSize, numClasses], dt)

    def crossEntropy(self, inp, tgt):
        x, shape, dt = self._get(inp)
        t = self.array(tgt)
        B, C = t.size, shape[-1]
        out = np.empty(B, np.float32)
        lib().or_cross_entropy(fp(x), fp(t), fp(out), B, C)
        return self._reg(out, [B], dt)

    def crossEntropyBackward(self, go, inp, tgt, reduction):
        g = self.array(go)
        x, shape, dt = self._get(inp)
        t = self.array(tgt)
        B, C = t.size, shape[-1]
        scale = 1.0 / max(1, B) if reduction == "mean" else 1.0
        out = np.empty(B * C, np.float32)
        lib().or_cross_entropy_backward(fp(g), 1 if g.size == 1 else 0, fp(x), fp(t), fp(out), B, C, scale)
        return self._reg(out, [B, C], dt)

    # ---- conv / pool / norm ----------------------------------------------
    def conv2d(self, inp, weight, bias, stride, padding, dilation, groups):
        x, sx, dt = self._get(inp)
        w, sw, _ = self._get(weight)
        p = conv_params(sx, sw, stride, padding)
        p.groups = int(groups)
        b = np.array(bias if bias is not None else [0.0] * sw[0], np.float32)
        out = np.empty(p.N * p.Cout * p.OH * p.OW, np.float32)
        lib().or_conv2d(fp(x), fp(w), fp(b), fp(out), ctypes.byref(p))
        return self._reg(out, [p.N, p.Cout, p.OH, p.OW], dt)

    def conv2dInputBackward(self, go, weight, inputShape, gradOutputShape, stride, padding):
        g, _, dt = self._get(go)
        w, sw, _ = self._get(weight)
        p = conv_params(inputShape, [gradOutputShape[1], inputShape[1], sw[2], sw[3]], stride, padding)
        p.OH, p.OW = gradOutputShape[2], gradOutputShape[3]
        out = np.empty(_prod(inputShape), np.float32)
        lib().or_conv2d_input_backward(fp(g), fp(w), fp(out), ctypes.byref(p))
        return self._reg(out, list(inputShape), dt)

    def conv2dWeightBackward(self, go, inp, weightShape, gradOutputShape, inputShape, stride, padding):
        g, _, dt = self._get(go)
        x = self.array(inp)
        p = conv_params(inputShape, weightShape, stride, padding)
        p.OH, p.OW = gradOutputShape[2], gradOutputShape[3]
        out = np.empty(_prod(weightShape), np.float32)
        lib().or_conv2d_weight_backward(fp(g), fp(x), fp(out), ctypes.byref(p))
        return self._reg(out, list(weightShape), dt)

    def conv2dBiasBackward(self, go, outCh, gradOutputShape):
        g, _, dt = self._get(go)
        N, _, OH, OW = gradOutputShape
        out = np.empty(outCh, np.float32)
        lib().or_conv2d_bias_backward(fp(g), fp(out), N, outCh, OH, OW)
        return self._reg(out, [outCh], dt)

    def maxPool2d(self, inp, kernelSize, stride, padding, dilation):
        x, sx, dt = self._get(inp)
        p = pool_params(sx, kernelSize, stride, padding, dilation)
        out = np.empty(p.N * p.C * p.OH * p.OW, np.float32)
        lib().or_max_pool2d(fp(x), fp(out), ip(None), ctypes.byref(p))
        return self._reg(out, [p.N, p.C, p.OH, p.OW], dt)

    def maxPool2dWithIndices(self, inp, kernelSize, stride, padding, dilation):
        x, sx, dt = self._get(inp)
        p = pool_params(sx, kernelSize, stride, padding, dilation)
        out = np.empty(p.N * p.C * p.OH * p.OW, np.float32)
        idx = np.empty(out.size, np.int32)
        lib().or_max_pool2d(fp(x), fp(out), ip(idx), ctypes.byref(p))
        shp = [p.N, p.C, p.OH, p.OW]
        return [self._reg(out, shp, dt), self._reg(idx.astype(np.float32), shp, "int32")]

    def maxPool2dBackward(self, go, indices, inputShape, kernelSize, stride, padding, dilation):
        g, so, dt = self._get(go)
        idx = self.array(indices).astype(np.int32)
        p = pool_params(inputShape, kernelSize, stride, padding, dilation)
        out = np.empty(_prod(inputShape), np.float32)
        lib().or_max_pool2d_backward(fp(g), ip(idx), fp(out), ctypes.byref(p))
        return self._reg(out, list(inputShape), dt)

    def _nc_s(self, shape):
        if len(shape) < 2:
            raise RuntimeError("batch_norm needs at least 2D input")
        return shape[0], shape[1], _prod(shape[2:])

    def batchNorm(self, inp, weight, bias, runningMean, runningVar, eps):
        x, sx, dt = self._get(inp)
        N, C, S = self._nc_s(sx)
        g = lambda t: self.array(t) if t is not None else None  # noqa: E731
        out = np.empty_like(x)
        lib().or_batchnorm_eval(fp(x), fp(g(weight)), fp(g(bias)), fp(g(runningMean)), fp(g(runningVar)), fp(out),
                                N, C, S, float(eps))
        return self._reg(out, sx, dt)

    def batchNormTrain(self, inp, weight, bias, runningMean, runningVar, eps, momentum):
        """New entry: returns [y, save_mean, save_invstd]; updates running stats."""
        x, sx, dt = self._get(inp)
        N, C, S = self._nc_s(sx)
        g = lambda t: self.array(t) if t is not None else None  # noqa: E731
        y = np.empty_like(x)
        sm = np.empty(C, np.float32)
        si = np.empty(C, np.float32)
        lib().or_batchnorm_train(fp(x), fp(g(weight)), fp(g(bias)), fp(g(runningMean)), fp(g(runningVar)), fp(y),
                                 fp(sm), fp(si), N, C, S, float(eps), float(momentum))
        return [self._reg(y, sx, dt), self._reg(sm, [C], dt), self._reg(si, [C], dt)]

    def batchNormBackward(self, go, inp, weight, saveMean, saveInvstd):
        """New entry: returns [dx, dweight, dbias] (PyTorch rule)."""
        dy, sx, dt = self._get(go)
        x = self.array(inp)
        N, C, S = self._nc_s(sx)
        w = self.array(weight) if weight is not None else None
        dx = np.empty_like(x)
        dw = np.empty(C, np.float32)
        db = np.empty(C, np.float32)
        lib().or_batchnorm_backward(fp(dy), fp(x), fp(w), fp(self.array(saveMean)), fp(self.array(saveInvstd)),
                                    fp(dx), fp(dw), fp(db), N, C, S)
        return [self._reg(dx, sx, dt), self._reg(dw, [C], dt), self._reg(db, [C], dt)]

    def layerNorm(self, inp, normalizedShape, gamma, beta, eps):
        x, sx, dt = self._get(inp)
        D = _prod(normalizedShape)
        rows = x.size // max(1, D)
        g = self.array(gamma) if gamma is not None else None
        b = self.array(beta) if beta is not None else None
        out = np.empty_like(x)
        lib().or_layernorm(fp(x), fp(g), fp(b), fp(out), fp(None), fp(None), rows, D, float(eps))
        return self._reg(out, sx, dt)

    def layerNormForward(self, inp, normalizedShape, gamma, beta, eps):
        """New entry: returns [y, mean, rstd] with per-row statistics."""
        x, sx, dt = self._get(inp)
        D = _prod(normalizedShape)
        rows = x.size // max(1, D)
        g = self.array(gamma) if gamma is not None else None
        b = self.array(beta) if beta is not None else None
        out = np.empty_like(x)
        mean = np.empty(rows, np.float32)
        rstd = np.empty(rows, np.float32)
        lib().or_layernorm(fp(x), fp(g), fp(b), fp(out), fp(mean), fp(rstd), rows, D, float(eps))
        return [self._reg(out, sx, dt), self._reg(mean, [rows], dt), self._reg(rstd, [rows], dt)]

    def layerNormBackward(self, go, inp, normalizedShape, gamma, saveMean, saveRstd):
        """New entry: returns [dx, dgamma, dbeta] (PyTorch rule)."""
        dy, sx, dt = self._get(go)
        x = self.array(inp)
        D = _prod(normalizedShape)
        rows = x.size // max(1, D)
        g = self.array(gamma) if gamma is not None else None
        dx = np.empty_like(x)
        dg = np.empty(D, np.float32)
        db = np.empty(D, np.float32)
        lib().or_layernorm_backward(fp(dy), fp(x), fp(g), fp(self.array(saveMean)), fp(self.array(saveRstd)),
                                    fp(dx), fp(dg), fp(db), rows, D)
        nshape = [int(s) for s in normalizedShape]
        return [self._reg(dx, sx, dt), self._reg(dg, nshape, dt), self._reg(db, nshape, dt)]

    # ---- optimizer steps (in place) --------------------------------------
    def _check4(self, *ids):
        arrs = [self.array(i) for i in ids]
        if any(a.size != arrs[0].size for a in arrs):
            raise RuntimeError("optimizer step: tensor lengths must match")
        return arrs

    def adamWStep(self, p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        P, G, Mm, V = self._check4(p, g, m, v)
        lib().or_adamw_step(fp(P), fp(G), fp(Mm), fp(V), P.size, lr, b1, b2, eps, wd, stepSize, invSqrtBc2)

    def adamStep(self, p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        P, G, Mm, V = self._check4(p, g, m, v)
        lib().or_adam_step(fp(P), fp(G), fp(Mm), fp(V), P.size, lr, b1, b2, eps, wd, stepSize, invSqrtBc2)

    def sgdStep(self, p, g, buf, lr, momentum, wd, dampening, nesterov):
        P, G, B = self._check4(p, g, buf)
        lib().or_sgd_step(fp(P), fp(G), fp(B), P.size, lr, momentum, wd, dampening, 1 if nesterov else 0)

    def adamWStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        for p, g, m, v in zip(ps, gs, ms, vs):
            self.adamWStep(p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2)

    def adamStepMulti(self, ps, gs, ms, vs, lr, b1, b2, eps, wd, stepSize, invSqrtBc2):
        for p, g, m, v in zip(ps, gs, ms, vs):
            self.adamStep(p, g, m, v, lr, b1, b2, eps, wd, stepSize, invSqrtBc2)

    def sgdStepMulti(self, ps, gs, bufs, lr, momentum, wd, dampening, nesterov):
        for p, g, b in zip(ps, gs, bufs):
            self.sgdStep(p, g, b, lr, momentum, wd, dampening, nesterov)

    def rmspropStep(self, p, g, squareAvg, momentumBuf, lr, alpha, eps, weightDecay, momentum):
        P, G, S, B = self._check4(p, g, squareAvg, momentumBuf)
        lib().or_rmsprop_step(fp(P), fp(G), fp(S), fp(B), P.size, lr, alpha, eps, weightDecay, momentum)

    def adagradStep(self, p, g, sumSquares, lr, eps, weightDecay):
        P, G, S = self._check4(p, g, sumSquares)
        lib().or_adagrad_step(fp(P), fp(G), fp(S), P.size, lr, eps, weightDecay)

    def adamaxStep(self, p, g, expAvg, expInf, lr, b1, b2, eps, wd, stepSize, biasCorrection1):
        P, G, M, U = self._check4(p, g, expAvg, expInf)
        lib().or_adamax_step(fp(P), fp(G), fp(M), fp(U), P.size, lr, b1, b2, eps, wd, stepSize, biasCorrection1)

    def nadamStep(self, p, g, expAvg, expAvgSq, lr, b1, b2, eps, wd, stepSize, mu):
        P, G, M, V = self._check4(p, g, expAvg, expAvgSq)
        lib().or_nadam_step(fp(P), fp(G), fp(M), fp(V), P.size, lr, b1, b2, eps, wd, stepSize, mu)

    def radamStep(self, p, g, expAvg, expAvgSq, lr, b1, b2, eps, wd, stepSize, beta1PowT, beta2PowT, stepCount=0):
        P, G, M, V = self._check4(p, g, expAvg, expAvgSq)
        lib().or_radam_step(fp(P), fp(G), fp(M), fp(V), P.size, lr, b1, b2, eps, wd, stepSize, beta1PowT, beta2PowT,
                            int(stepCount))

    def rmspropStepMulti(self, ps, gs, sqs, mbs, lr, alpha, eps, weightDecay, momentum):
        for a in zip(ps, gs, sqs, mbs):
            self.rmspropStep(*a, lr, alpha, eps, weightDecay, momentum)

    def adagradStepMulti(self, ps, gs, sums, lr, eps, weightDecay):
        for a in zip(ps, gs, sums):
            self.adagradStep(*a, lr, eps, weightDecay)

    def adamaxStepMulti(self, ps, gs, ms, us, *hp):
        for a in zip(ps, gs, ms, us):
            self.adamaxStep(*a, *hp)

    def nadamStepMulti(self, ps, gs, ms, vs, *hp):
        for a in zip(ps, gs, ms, vs):
            self.nadamStep(*a, *hp)

    def radamStepMulti(self, ps, gs, ms, vs, *hp):
        for a in zip(ps, gs, ms, vs):
            self.radamStep(*a, *hp)

    # ---- conv2d with a bias tensor; bulk bytes ----------------------------
    def conv2dDevBias(self, inp, weight, bias, stride, padding, dilation, groups):
        blist = self.array(bias).tolist() if bias is not None else None
        return self.conv2d(inp, weight, blist, stride, padding, dilation, groups)

    def toBytes(self, tid, fmt: str = "float32") -> bytes:
        x = self.array(tid)
        if fmt == "int64":
            return np.trunc(x).astype("<i8").tobytes()
        return x.astype("<f4").tobytes()

    def fromBytes(self, data, shape, dtype, fmt: str = "float32"):
        if fmt == "int64":
            arr = np.frombuffer(bytes(data), dtype="<i8").astype(np.float32)
        else:
            arr = np.frombuffer(bytes(data), dtype="<f4").astype(np.float32)
        if arr.size != _prod(shape):
            raise RuntimeError(f"fromBytes: {arr.size} values for shape {list(shape)}")
        return self._reg(arr, shape, dtype)

    # shapeOps.ts select / cat (runtime.ts:876-897): the reference DataLoader's
    # per-sample path (TensorDataset indexing, then stack = unsqueeze + cat);
    # copies, as every reference shape op
    def select(self, tid, dim, index):
        x, shape, dt = self._get(tid)
        d = dim + len(shape) if dim < 0 else dim
        i = index + shape[d] if index < 0 else index
        if not 0 <= i < shape[d]:
            raise RuntimeError(f"select: index {index} out of range for dim {dim} of size {shape[d]}")
        out = np.take(x.reshape(shape), i, axis=d)
        return self._reg(np.ascontiguousarray(out).reshape(-1), list(out.shape), dt)

    def cat(self, ids, dim):
        arrs = [self._get(t) for t in ids]
        d = dim + len(arrs[0][1]) if dim < 0 else dim
        out = np.concatenate([a.reshape(sh) for a, sh, _ in arrs], axis=d)
        return self._reg(out.reshape(-1), list(out.shape), arrs[0][2])

    def gatherRows(self, tid, rows):
        x, shape, dt = self._get(tid)
        rows = [int(r) for r in rows]
        if any(r < 0 or r >= shape[0] for r in rows):
            raise RuntimeError("gatherRows: index out of bounds for dimension 0")
        return self._reg(x.reshape(shape[0], -1)[rows].reshape(-1), [len(rows)] + list(shape[1:]), dt)

    # ---- readback / lifetime ---------------------------------------------
    def toList(self, tid):
        x, _, dt = self._get(tid)
        if dt == "bool":
            return [1 if v != 0 else 0 for v in x.tolist()]
        if dt.startswith("int") or dt.startswith("uint"):
            return [int(math.trunc(v)) for v in x.tolist()]
        return x.tolist()

    def destroy(self, tid) -> None:
        self._t.pop(int(tid), None)
