"""VGG-11-BN training step driver on the pointer-level C ABI.

The reference trains through its Python autograd, one runtime call per op
(python/torch/autograd_engine.py:45-161) with ~15 composed dispatches per
BatchNorm, and cannot run this model's backward at all (the BN backward throws
for W != C, python/torch/autograd_rules.py:1082; max-pool has no backward,
python/torch/tensor_nn_ops.py:57-72).  Here the step is a fixed sequence of
fused kernels on preallocated HBM buffers:

  forward   per block: conv3x3 (+bias) -> BN (batch stats, running stats) + ReLU
            -> [2x2 max-pool with indices]; then linear 512->10 and the
            cross-entropy mean, both left in HBM
  backward  CE -> linear -> per block: [pool backward] -> BN backward with the
            ReLU mask folded in -> conv bias / weight / data gradients
  update    data-parallel: gradient all-reduce (NCCL, bucketed, issued as soon
            as each block's gradients are final); one fused SGD-momentum launch
            over all parameters with the 1/world averaging folded in

The whole step is captured once into a CUDA graph and replayed.  Semantics:
PyTorch's (SGD momentum 0.9 with weight decay 5e-4, dampening 0; BN momentum
0.1, eps 1e-5, unbiased running variance), which is what the reference's
modules and optimizers intend (python/torch/nn/modules.py:548-597,
python/torch/optim/__init__.py:158-205).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from ._lib import check

CFG = [64, "M", 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"]
NUM_CLASSES = 10


def _vp(x: int):
    return ctypes.c_void_p(int(x)) if x else None


def plan_blocks(cfg=CFG, in_ch: int = 3, size: int = 32) -> list[dict]:
    """One dict per conv block: cin, cout, H, W (the conv's spatial size) and
    whether a 2x2 max-pool follows."""
    blocks = []
    cin, H = in_ch, size
    i = 0
    while i < len(cfg):
        cout = cfg[i]
        pool = i + 1 < len(cfg) and cfg[i + 1] == "M"
        blocks.append({"cin": cin, "cout": cout, "H": H, "W": H, "pool": pool})
        cin = cout
        if pool:
            H //= 2
            i += 2
        else:
            i += 1
    return blocks


def plan_params(blocks: list[dict], feat: int) -> tuple[list, dict, int]:
    """Parameter specs (name, shape, init) in the order backward finishes
    them (fc first, conv1 last), their (offset, numel) in the flat buffers
    (each tensor starts on a 256-byte boundary) and the flat length."""
    specs = []
    specs.append(("fc.w", [NUM_CLASSES, feat], ("kaiming", feat)))
    specs.append(("fc.b", [NUM_CLASSES], ("bias", feat)))
    for li in reversed(range(len(blocks))):
        b = blocks[li]
        fan_in = b["cin"] * 9
        specs.append((f"bn{li}.g", [b["cout"]], ("const", 1.0)))
        specs.append((f"bn{li}.b", [b["cout"]], ("const", 0.0)))
        specs.append((f"conv{li}.b", [b["cout"]], ("bias", fan_in)))
        specs.append((f"conv{li}.w", [b["cout"], b["cin"], 3, 3], ("kaiming", fan_in)))
    offsets = {}
    off = 0
    for name, shape, _ in specs:
        n = int(np.prod(shape))
        offsets[name] = (off, n)
        off += (n + 63) // 64 * 64
    return specs, offsets, off


def init_params(specs: list, offsets: dict, flat_len: int, seed: int) -> np.ndarray:
    """The flat parameter buffer on the host: PyTorch's default Conv2d/Linear
    init (kaiming_uniform_ with a=sqrt(5), i.e. U(+-1/sqrt(fan_in)), for
    weights and biases), BN gamma 1 and beta 0; padding zero."""
    rng = np.random.default_rng(seed)
    host = np.zeros(flat_len, np.float32)
    for name, _, init in specs:
        o, n = offsets[name]
        if init[0] in ("kaiming", "bias"):
            bound = 1.0 / math.sqrt(init[1])
            host[o:o + n] = rng.uniform(-bound, bound, n)
        else:
            host[o:o + n] = init[1]
    return host


def plan_buckets(offsets: dict, nblocks: int, flat_len: int, bucket_bytes: int) -> list[tuple[int, int, str]]:
    """Split the flat gradient buffer into contiguous buckets of at least
    bucket_bytes (the last one takes the rest), each closing after the layer
    whose gradients end it: (start element, element count, layer key), keys
    "fc" and "blk<i>", in backward order.  Together the buckets cover
    [0, flat_len) exactly once."""
    buckets = []
    order = ["fc"] + [f"blk{li}" for li in reversed(range(nblocks))]
    ends = {"fc": offsets["fc.b"][0] + offsets["fc.b"][1]}
    for li in range(nblocks):
        o, n = offsets[f"conv{li}.w"]
        ends[f"blk{li}"] = o + n
    start = 0
    limit = max(1, bucket_bytes // 4)
    for key in order:
        end = ends[key]
        if end - start >= limit or key == order[-1]:
            buckets.append((start, (flat_len if key == order[-1] else end) - start, key))
            start = end
    return buckets


class VGG11BN:
    """Buffers, parameters and the step sequence of VGG-11-BN on 32x32 inputs."""

    def __init__(self, rt, batch: int, seed: int = 0, lr: float = 0.05, momentum: float = 0.9,
                 weight_decay: float = 5e-4, world: int = 1, comm=None, bucket_bytes: int = 8 << 20):
        self.rt, self.lib = rt, rt.lib
        self.B = int(batch)
        self.lr, self.momentum, self.wd = lr, momentum, weight_decay
        self.world = int(world)
        self.comm = comm
        self.bucket_bytes = bucket_bytes
        self._allocs = []
        self.graph = None
        # ---- layer plan ----
        self.blocks = plan_blocks()
        last = self.blocks[-1]
        self.feat = last["cout"] * (last["H"] // 2) ** 2  # 512
        assert self.feat == 512

        # ---- parameters, gradients, momentum: one flat buffer each, laid out in
        # the order backward finishes them so gradient buckets close in
        # backward order ----
        specs, self.offsets, self.flat_len = plan_params(self.blocks, self.feat)
        self.param_specs = specs
        self.nparams = sum(int(np.prod(s)) for _, s, _ in specs)
        self.params = self._alloc(self.flat_len * 4)
        self.grads = self._alloc(self.flat_len * 4)
        self.moms = self._alloc(self.flat_len * 4)
        self._h2d(self.params, init_params(specs, self.offsets, self.flat_len, seed))
        check(self.lib.tp_memset(_vp(self.grads), 0, self.flat_len * 4))
        check(self.lib.tp_memset(_vp(self.moms), 0, self.flat_len * 4))

        # BN running stats and saved batch statistics
        for li, b in enumerate(self.blocks):
            C = b["cout"]
            b["rm"] = self._alloc(C * 4)
            b["rv"] = self._alloc(C * 4)
            self._h2d(b["rm"], np.zeros(C, np.float32))
            self._h2d(b["rv"], np.ones(C, np.float32))
            b["mean"] = self._alloc(C * 4)
            b["invstd"] = self._alloc(C * 4)

        # ---- activations ----
        Bn = self.B
        self.x = self._alloc(Bn * 3 * 32 * 32 * 4)
        self.y = self._alloc(Bn * 4)
        max_act = 0
        for b in self.blocks:
            n = Bn * b["cout"] * b["H"] * b["W"]
            max_act = max(max_act, n, Bn * b["cin"] * b["H"] * b["W"])
            b["z"] = self._alloc(n * 4)  # conv output (BN input)
            b["a"] = self._alloc(n * 4)  # BN + ReLU output
            if b["pool"]:
                m = n // 4
                b["p"] = self._alloc(m * 4)
                b["idx"] = self._alloc(m * 4)
            b["out"] = b["p"] if b["pool"] else b["a"]
        self.logits = self._alloc(Bn * NUM_CLASSES * 4)
        self.dlogits = self._alloc(Bn * NUM_CLASSES * 4)
        self.loss_rows = self._alloc(Bn * 4)
        self.loss = self._alloc(4)
        self.dfeat = self._alloc(Bn * self.feat * 4)
        self.gbuf = [self._alloc(max_act * 4), self._alloc(max_act * 4)]

        # ---- optimizer group: every parameter tensor, fused SGD ----
        names = [n for n, _, _ in specs]
        ptr = lambda base: (ctypes.c_void_p * len(names))(*[base + 4 * self.offsets[n][0] for n in names])  # noqa
        numels = (ctypes.c_int64 * len(names))(*[self.offsets[n][1] for n in names])
        g = ctypes.c_int64(0)
        check(self.lib.tpk_group_create(len(names), ptr(self.params), ptr(self.grads), ptr(self.moms), None, numels,
                                        ctypes.byref(g)))
        self.group = g.value

        # gradient buckets (contiguous ranges of the flat gradient buffer)
        self._plan_buckets()

    # ---- helpers --------------------------------------------------------------------
    def _alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(self.lib.tp_alloc(int(nbytes), ctypes.byref(p)))
        self._allocs.append(p.value)
        return int(p.value)

    def _h2d(self, dst: int, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr, np.float32)
        check(self.lib.tp_memcpy_h2d(_vp(dst), arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes))
        self.rt.synchronize()

    def p(self, name: str) -> int:
        return self.params + 4 * self.offsets[name][0]

    def g(self, name: str) -> int:
        return self.grads + 4 * self.offsets[name][0]

    def _plan_buckets(self) -> None:
        self.buckets = plan_buckets(self.offsets, len(self.blocks), self.flat_len, self.bucket_bytes)
        self.bucket_after = {b[2]: b for b in self.buckets}

    # ---- the step ----------------------------------------------------------------------
    def _forward(self) -> None:
        L = self.lib
        Bn = self.B
        x = self.x
        for li, b in enumerate(self.blocks):
            C, H, W = b["cout"], b["H"], b["W"]
            check(L.tpk_conv2d_fwd(_vp(x), _vp(self.p(f"conv{li}.w")), _vp(self.p(f"conv{li}.b")), _vp(b["z"]), Bn,
                                   b["cin"], H, W, C, 3, 3, 1, 1, 1, 1))
            check(L.tpk_bn_train(_vp(b["z"]), _vp(self.p(f"bn{li}.g")), _vp(self.p(f"bn{li}.b")), _vp(b["rm"]),
                                 _vp(b["rv"]), _vp(b["a"]), _vp(b["mean"]), _vp(b["invstd"]), Bn, C, H * W, 1e-5,
                                 0.1, 1))
            if b["pool"]:
                check(L.tpk_maxpool_fwd(_vp(b["a"]), _vp(b["p"]), _vp(b["idx"]), Bn, C, H, W, 2, 2, 0))
            x = b["out"]
        self.feat_ptr = x
        check(L.tpk_gemm(_vp(x), 0, _vp(self.p("fc.w")), 1, _vp(self.logits), Bn, NUM_CLASSES, self.feat,
                         _vp(self.p("fc.b"))))
        check(L.tpk_cross_entropy_mean(_vp(self.logits), _vp(self.y), _vp(self.loss_rows), _vp(self.loss), Bn,
                                       NUM_CLASSES))

    def _reduce(self, key: str) -> None:
        if self.comm is not None and key in self.bucket_after:
            start, count, _ = self.bucket_after[key]
            self.comm.allreduce_async(self.grads + 4 * start, count)

    def _backward(self) -> None:
        L = self.lib
        Bn = self.B
        check(L.tpk_cross_entropy_backward(_vp(self.logits), _vp(self.y), _vp(self.dlogits), Bn, NUM_CLASSES,
                                           1.0 / Bn))
        check(L.tpk_gemm(_vp(self.dlogits), 1, _vp(self.feat_ptr), 0, _vp(self.g("fc.w")), NUM_CLASSES, self.feat,
                         Bn, None))
        check(L.tpk_channel_sum(_vp(self.dlogits), Bn, NUM_CLASSES, 1, _vp(self.g("fc.b"))))
        check(L.tpk_gemm(_vp(self.dlogits), 0, _vp(self.p("fc.w")), 0, _vp(self.dfeat), Bn, self.feat, NUM_CLASSES,
                         None))
        self._reduce("fc")
        gout = self.dfeat
        buf = 0
        for li in reversed(range(len(self.blocks))):
            b = self.blocks[li]
            C, H, W = b["cout"], b["H"], b["W"]
            if b["pool"]:
                da = self.gbuf[buf]
                buf ^= 1
                check(L.tpk_maxpool_bwd(_vp(gout), _vp(b["idx"]), _vp(da), Bn, C, H, W, 2, 2, 0))
            else:
                da = gout
            dz = self.gbuf[buf]
            buf ^= 1
            check(L.tpk_bn_backward(_vp(da), _vp(b["z"]), _vp(b["a"]), _vp(self.p(f"bn{li}.g")), _vp(b["mean"]),
                                    _vp(b["invstd"]), _vp(dz), _vp(self.g(f"bn{li}.g")), _vp(self.g(f"bn{li}.b")), Bn,
                                    C, H * W))
            check(L.tpk_channel_sum(_vp(dz), Bn, C, H * W, _vp(self.g(f"conv{li}.b"))))
            xin = self.x if li == 0 else self.blocks[li - 1]["out"]
            check(L.tpk_conv2d_wgrad(_vp(dz), _vp(xin), _vp(self.g(f"conv{li}.w")), Bn, b["cin"], H, W, C, 3, 3, 1,
                                     1, 1, 1))
            self._reduce(f"blk{li}")
            if li > 0:
                dx = self.gbuf[buf]
                buf ^= 1
                check(L.tpk_conv2d_dgrad(_vp(dz), _vp(self.p(f"conv{li}.w")), _vp(dx), Bn, b["cin"], H, W, C, 3, 3, 1,
                                         1, 1, 1))
                gout = dx

    def _update(self) -> None:
        if self.comm is not None:
            self.comm.wait()
        check(self.lib.tpk_sgd_group(self.group, self.lr, self.momentum, self.wd, 0.0, 0, 1.0 / self.world))

    def step_eager(self) -> None:
        self._forward()
        self._backward()
        self._update()

    def capture(self) -> None:
        """Run the step once eagerly (sizes the scratch), then capture it."""
        self.step_eager()
        self.rt.synchronize()
        check(self.lib.tp_graph_begin())
        try:
            self.step_eager()
        finally:
            gid = ctypes.c_int64(0)
            check(self.lib.tp_graph_end(ctypes.byref(gid)))
        self.graph = gid.value

    def step(self) -> None:
        if self.graph is not None:
            check(self.lib.tp_graph_launch(self.graph))
        else:
            self.step_eager()

    # ---- data / readback ----------------------------------------------------------------
    def set_batch_device(self, x_host_ptr: int, y_host_ptr: int) -> None:
        """Copy one batch from (pinned) host memory into the input buffers."""
        check(self.lib.tp_memcpy_h2d(_vp(self.x), _vp(x_host_ptr), self.B * 3 * 32 * 32 * 4))
        check(self.lib.tp_memcpy_h2d(_vp(self.y), _vp(y_host_ptr), self.B * 4))

    def read_loss(self) -> float:
        out = np.zeros(1, np.float32)
        check(self.lib.tp_memcpy_d2h(out.ctypes.data_as(ctypes.c_void_p), _vp(self.loss), 4))
        return float(out[0])

    def read(self, ptr: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        check(self.lib.tp_memcpy_d2h(out.ctypes.data_as(ctypes.c_void_p), _vp(ptr), n * 4))
        return out

    def param_array(self, name: str) -> np.ndarray:
        o, n = self.offsets[name]
        return self.read(self.params + 4 * o, n)

    def close(self) -> None:
        if self.graph is not None:
            self.lib.tp_graph_destroy(self.graph)
            self.graph = None
        self.lib.tpk_group_destroy(self.group)
        for p in self._allocs:
            self.lib.tp_free(_vp(p))
        self._allocs = []

    # algorithmic work of one step at this batch (for the roofline)
    def step_flops(self) -> float:
        f = 0.0
        for li, b in enumerate(self.blocks):
            macs = self.B * b["cout"] * b["H"] * b["W"] * b["cin"] * 9
            f += 2 * macs * (3 if li > 0 else 2)  # fwd + wgrad (+ dgrad except layer 1)
        f += 2 * self.B * self.feat * NUM_CLASSES * 3
        return f
