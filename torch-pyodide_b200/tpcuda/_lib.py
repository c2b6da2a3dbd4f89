"""ctypes binding of libtpcuda.so (include/tpcuda.h).

The library is built in-tree by ``tpcuda.build.build()`` (nvcc, sm_100a) next
to this file.  There is no fallback: if the shared library is missing or no
CUDA device is visible, loading raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtpcuda.so")

MAX_DIMS = 8

DTYPES = ["float32", "float16", "bfloat16", "int8", "int16", "int32", "int64", "uint8", "uint16", "uint32",
          "uint64", "bool"]
DTYPE_CODE = {name: i for i, name in enumerate(DTYPES)}

# status codes
TP_OK = 0


class Handle(ctypes.Structure):
    """tp_handle: the reference TensorHandle {id, shape, dtype}."""

    _fields_ = [("id", ctypes.c_int64), ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("shape", ctypes.c_int64 * MAX_DIMS)]

    def to_dict(self) -> dict:
        return {"id": int(self.id), "shape": [int(self.shape[i]) for i in range(self.ndim)],
                "dtype": DTYPES[self.dtype]}


class TpError(RuntimeError):
    """A non-zero status from libtpcuda (the reference's JS Error)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


I64 = ctypes.c_int64
I32 = ctypes.c_int32
F32 = ctypes.c_float
P = ctypes.c_void_p
HP = ctypes.POINTER(Handle)
I64P = ctypes.POINTER(ctypes.c_int64)
I32P = ctypes.POINTER(ctypes.c_int32)
F32P = ctypes.POINTER(ctypes.c_float)
PP = ctypes.POINTER(ctypes.c_void_p)
INT = ctypes.c_int

# name -> argtypes (restype int unless listed in _RESTYPE)
SIGNATURES: dict[str, list] = {
    "tp_init": [INT],
    "tp_is_available": [],
    "tp_device_count": [ctypes.POINTER(INT)],
    "tp_last_error": [],
    "tp_synchronize": [],
    "tp_get_stream": [PP],
    "tp_aux_fork": [],
    "tp_aux_return": [],
    "tp_aux_record": [INT],
    "tp_main_wait": [INT],
    "tp_aux_join": [],
    "tp_side_fork": [],
    "tp_side_return": [],
    "tp_side_join": [],
    "tp_memory_allocated": [I64P],
    "tp_memory_reserved": [I64P],
    "tp_device_name": [ctypes.c_char_p, INT],
    "tp_kernel_launches": [I64P],
    "tp_tensor_from_data": [P, I64P, INT, INT, HP],
    "tp_to_host": [I64, P, I64],
    "tp_destroy": [I64],
    "tp_meta": [I64, HP],
    "tp_device_ptr": [I64, PP],
    "tp_alloc": [I64, PP],
    "tp_free": [P],
    "tp_memcpy_h2d": [P, P, I64],
    "tp_memcpy_d2h": [P, P, I64],
    "tp_memcpy_d2d": [P, P, I64],
    "tp_to_bytes": [I64, P, I64, INT],
    "tp_from_bytes": [P, I64, INT, I64P, INT, INT, HP],
    "tp_host_alloc": [I64, PP],
    "tp_host_free": [P],
    "tp_tensor_from_host_async": [P, I64P, INT, INT, INT, HP, I64P],
    "tp_ticket_use": [I64],
    "tp_ticket_wait": [I64],
    "tp_gather_rows": [I64, I64P, I64, HP],
    "tp_conv2d_dev_bias": [I64, I64, I64, I64P, INT, I64P, INT, I64P, INT, INT, HP],
    "tp_rmsprop_step": [I64, I64, I64, I64, F32, F32, F32, F32, F32],
    "tp_adagrad_step": [I64, I64, I64, F32, F32, F32],
    "tp_adamax_step": [I64, I64, I64, I64] + [F32] * 7,
    "tp_nadam_step": [I64, I64, I64, I64] + [F32] * 7,
    "tp_radam_step": [I64, I64, I64, I64] + [F32] * 8 + [I64],
    "tp_rmsprop_step_multi": [I64P, I64P, I64P, I64P, INT, F32, F32, F32, F32, F32],
    "tp_adagrad_step_multi": [I64P, I64P, I64P, INT, F32, F32, F32],
    "tp_adamax_step_multi": [I64P, I64P, I64P, I64P, INT] + [F32] * 7,
    "tp_nadam_step_multi": [I64P, I64P, I64P, I64P, INT] + [F32] * 7,
    "tp_radam_step_multi": [I64P, I64P, I64P, I64P, INT] + [F32] * 8 + [I64],
    "tp_memset": [P, INT, I64],
    "tp_full": [I64P, INT, INT, F32, HP],
    "tp_full_like": [I64, INT, F32, HP],
    "tp_fill": [I64, F32, HP],
    "tp_set_seed": [ctypes.c_uint32],
    "tp_random": [I64P, INT, INT, INT, F32, F32, HP],
    "tp_binary": [INT, I64, I64, HP],
    "tp_add": [I64, I64, HP],
    "tp_sub": [I64, I64, HP],
    "tp_mul": [I64, I64, HP],
    "tp_div": [I64, I64, HP],
    "tp_pow": [I64, I64, HP],
    "tp_gt": [I64, I64, HP],
    "tp_mul_scalar": [I64, F32, HP],
    "tp_unary": [INT, I64, HP],
    "tp_relu": [I64, HP],
    "tp_rsqrt": [I64, HP],
    "tp_neg": [I64, HP],
    "tp_reshape": [I64, I64P, INT, HP],
    "tp_transpose2d": [I64, HP],
    "tp_permute": [I64, I32P, INT, HP],
    "tp_expand": [I64, I64P, INT, HP],
    "tp_reduce_all": [I64, INT, HP],
    "tp_sum": [I64, HP],
    "tp_mean": [I64, HP],
    "tp_max": [I64, HP],
    "tp_reduce_dim": [I64, INT, INT, INT, HP],
    "tp_sum_dim": [I64, INT, INT, HP],
    "tp_mean_dim": [I64, INT, INT, HP],
    "tp_max_dim": [I64, INT, INT, HP, HP],
    "tp_argmax": [I64, HP],
    "tp_softmax": [I64, INT, HP],
    "tp_log_softmax": [I64, INT, HP],
    "tp_softmax_backward": [I64, I64, I64, I64, HP],
    "tp_log_softmax_backward": [I64, I64, I64, I64, HP],
    "tp_cross_entropy": [I64, I64, HP],
    "tp_cross_entropy_backward": [I64, I64, I64, INT, HP],
    "tp_set_gemm_path": [INT],
    "tp_set_pdl": [INT],
    "tp_gemm_status": [ctypes.POINTER(INT), INT],
    "tp_wait_probe": [I64],
    "tp_set_gemm_kmax": [INT],
    "tp_set_gemm_twocta": [INT],
    "tp_set_bn_flow": [INT, INT, INT, INT],
    "tp_matmul": [I64, I64, HP],
    "tp_linear": [I64, I64, I64, HP],
    "tp_conv2d": [I64, I64, F32P, INT, I64P, INT, I64P, INT, I64P, INT, INT, HP],
    "tp_conv2d_input_backward": [I64, I64, I64P, I64P, I64P, INT, I64P, INT, HP],
    "tp_conv2d_weight_backward": [I64, I64, I64P, I64P, I64P, I64P, INT, I64P, INT, HP],
    "tp_conv2d_bias_backward": [I64, I64, I64P, HP],
    "tp_max_pool2d": [I64, I64P, INT, I64P, INT, I64P, INT, I64P, INT, HP],
    "tp_max_pool2d_with_indices": [I64, I64P, INT, I64P, INT, I64P, INT, I64P, INT, HP, HP],
    "tp_max_pool2d_backward": [I64, I64, I64P, I64P, INT, I64P, INT, I64P, INT, I64P, INT, HP],
    "tp_batch_norm": [I64, I64, I64, I64, I64, F32, HP],
    "tp_batch_norm_train": [I64, I64, I64, I64, I64, F32, F32, INT, HP, HP, HP],
    "tp_batch_norm_backward": [I64, I64, I64, I64, I64, I64, HP, HP, HP],
    "tp_layer_norm": [I64, I64, I64, I64, F32, HP, HP, HP],
    "tp_layer_norm_backward": [I64, I64, I64, I64, I64, I64, HP, HP, HP],
    "tp_adamw_step": [I64, I64, I64, I64] + [F32] * 7,
    "tp_adam_step": [I64, I64, I64, I64] + [F32] * 7,
    "tp_sgd_step": [I64, I64, I64, F32, F32, F32, F32, INT],
    "tp_adamw_step_multi": [I64P, I64P, I64P, I64P, INT] + [F32] * 7,
    "tp_adam_step_multi": [I64P, I64P, I64P, I64P, INT] + [F32] * 7,
    "tp_sgd_step_multi": [I64P, I64P, I64P, INT, F32, F32, F32, F32, INT],
    "tpk_group_create": [INT, PP, PP, PP, PP, I64P, I64P],
    "tpk_group_create_lo": [INT, PP, PP, PP, PP, PP, I64P, I64P],
    "tpk_group_destroy": [I64],
    "tpk_adam_group": [I64, INT] + [F32] * 7,
    "tpk_sgd_group": [I64, F32, F32, F32, F32, INT, F32],
    "tpk_conv2d_fwd": [P, P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT, INT],
    "tpk_conv2d_dgrad": [P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT, INT],
    "tpk_conv2d_wgrad": [P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT, INT],
    "tpk_bn_train_nhwc": [P, P, P, P, P, P, P, P, I64, I64, F32, F32, INT],
    "tpk_bn_backward_nhwc": [P, P, P, P, P, P, P, P, P, P, I64, I64],
    "tpk_bn_train_pool_nhwc": [P] * 10 + [I64, I64, I64, I64, F32, F32, INT],
    "tpk_bn_backward_fused_nhwc": [P] * 11 + [I64, I64, I64, I64, INT],
    "tpk_channel_sum_nhwc": [P, I64, I64, P],
    "tpk_maxpool2x2_nhwc_fwd": [P, P, P, I64, I64, I64, I64],
    "tpk_maxpool2x2_nhwc_bwd": [P, P, P, I64, I64, I64, I64],
    "tpk_nchw_to_nhwc": [P, P, I64, I64, I64, I64, I64],
    "tpk_conv2d_fwd_nhwc": [P, P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT],
    "tpk_conv2d_dgrad_nhwc": [P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT],
    "tpk_conv2d_wgrad_nhwc": [P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT],
    "tpk_conv2d_fwd_nhwc_lo": [P, P, P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT],
    "tpk_conv2d_dgrad_nhwc_lo": [P, P, P, P, I64, I64, I64, I64, I64, INT, INT, INT, INT, INT],
    "tpk_tf32_lo": [P, P, I64],
    "tpk_channel_sum": [P, I64, I64, I64, P],
    "tpk_bn_train": [P, P, P, P, P, P, P, P, I64, I64, I64, F32, F32, INT],
    "tpk_bn_backward": [P, P, P, P, P, P, P, P, P, I64, I64, I64],
    "tpk_maxpool_fwd": [P, P, P, I64, I64, I64, I64, INT, INT, INT],
    "tpk_maxpool_bwd": [P, P, P, I64, I64, I64, I64, INT, INT, INT],
    "tpk_gemm": [P, INT, P, INT, P, I64, I64, I64, P],
    "tpk_cross_entropy_mean": [P, P, P, P, I64, I64],
    "tpk_cross_entropy_mean_noalloc": [P, P, P, I64, I64],
    "tpk_linear_cross_entropy_step": [P, P, P, P, P, P, P, P, P, P, I64, I64, I64, F32],
    "tpk_cross_entropy_backward": [P, P, P, I64, I64, F32],
    "tpk_fill": [P, I64, F32],
    "tp_comm_unique_id": [ctypes.c_char_p, INT],
    "tp_set_comm_priority": [INT],
    "tp_comm_init": [INT, INT, ctypes.c_char_p, INT],
    "tp_comm_allreduce_async": [P, I64],
    "tp_comm_wait": [],
    "tp_comm_sync": [INT],
    "tp_comm_destroy": [],
    "tp_comm_info": [ctypes.POINTER(INT), ctypes.POINTER(INT)],
    "tp_graph_begin": [],
    "tp_graph_end": [I64P],
    "tp_graph_launch": [I64],
    "tp_graph_destroy": [I64],
}

_RESTYPE = {"tp_last_error": ctypes.c_char_p}

_lib = None


def load(path: str | None = None):
    """Load libtpcuda.so and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(f"libtpcuda.so not found at {p}; build it with tpcuda.build.build()")
    L = ctypes.CDLL(p)
    for name, args in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    _lib = L
    return L


def check(status: int) -> None:
    if status != TP_OK:
        msg = _lib.tp_last_error().decode("utf-8", "replace") if _lib is not None else "libtpcuda error"
        raise TpError(status, msg)


def i64arr(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)
