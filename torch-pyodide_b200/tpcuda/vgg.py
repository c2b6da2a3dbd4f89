"""VGG-11-BN training step driver on the pointer-level C ABI.

The reference trains through its Python autograd, one runtime call per op
(python/torch/autograd_engine.py:45-161) with ~15 composed dispatches per
BatchNorm, and cannot run this model's backward at all (the BN backward throws
for W != C, python/torch/autograd_rules.py:1082; max-pool has no backward,
python/torch/tensor_nn_ops.py:57-72).  Here the step is a fixed sequence of
fused kernels on preallocated HBM buffers:

  forward   per block: conv3x3 (+bias) -> BN (batch stats, running stats) + ReLU
            -> [2x2 max-pool with indices]; then the classifier head in one
            launch: linear 512->10, the cross-entropy mean (left in HBM) and
            the gradients of both (fc weight / bias, the feature gradient)
  backward  per block: [pool backward] -> BN backward with the
            ReLU mask folded in -> conv bias / weight / data gradients
  update    data-parallel: gradient all-reduce (NCCL, bucketed, issued as soon
            as each block's gradients are final); fused SGD-momentum with the
            1/world averaging folded in: data-parallel channels-last steps update
            each bucket as soon as its all-reduce is done and its block's data
            gradient (the last reader of its filters) has run, beside the rest of
            the backward on a side stream; one GPU (unless early_update=True)
            and the NCHW cross-check update everything in one launch at the end

Activations are channels-last ([N][H][W][C], layout="nhwc", the default):
each implicit-GEMM tile of the convolutions is then one TMA box, and the
norm / pool passes move 16-byte vectors of 4 channels.  The input batch
arrives NCHW and is converted on the device into a channels-last buffer whose
3 channels are zero-padded to 4 (one 16-byte vector per pixel, the form the
first layer's CUDA-core kernels read); the first conv's filters are stored
with the same padding, their padded channel stays exactly zero (zero input,
zero gradient, zero decay).  The other convs' filters are stored
[Cout][3][3][Cin]: the forward uses them as they are, the data gradient reads
them in place and the weight gradient writes that layout with contiguous
stores, so no filter is repacked per step.  layout="nchw" runs the same step
on the NCHW kernels of the per-op API, as a cross-check.

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


CIN0_PAD = 4  # channels of the first conv's input as stored channels-last


def plan_params(blocks: list[dict], feat: int, cin0_store: int = 3, khwc: bool = False) -> tuple[list, dict, int]:
    """Parameter specs (name, shape, init) in the order backward finishes
    them (fc first, conv1 last), their (offset, stored numel) in the flat
    buffers (each tensor starts on a 256-byte boundary) and the flat length.
    The first conv's filters are stored as [Cout][cin0_store][3][3] (input
    channels zero-padded when cin0_store > 3); with khwc the other convs'
    filters are stored [Cout][3][3][Cin] (see store_shape)."""
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
        n = int(np.prod(store_shape(name, shape, cin0_store, khwc)))
        offsets[name] = (off, n)
        off += (n + 63) // 64 * 64
    return specs, offsets, off


def store_shape(name: str, shape: list, cin0_store: int, khwc: bool = False) -> list:
    """Stored shape of a parameter: the first conv's filters may be padded
    ([Cout][cin0_store][3][3]); with khwc the other convs' filters are stored
    [Cout][KH][KW][Cin], the order the channels-last convolutions read them
    in place."""
    if name == "conv0.w":
        return [shape[0], cin0_store, shape[2], shape[3]] if cin0_store != shape[1] else list(shape)
    if khwc and name.startswith("conv") and name.endswith(".w"):
        return [shape[0], shape[2], shape[3], shape[1]]
    return list(shape)


def to_store(name: str, v: np.ndarray, shape: list, cin0_store: int, khwc: bool = False) -> np.ndarray:
    """A parameter's values in its logical (reference) layout -> stored layout (flat)."""
    st = store_shape(name, shape, cin0_store, khwc)
    if st == list(shape):
        return np.ascontiguousarray(v, np.float32).ravel()
    if name == "conv0.w":
        w = np.zeros(st, np.float32)
        w[:, :shape[1]] = v.reshape(shape)
        return w.ravel()
    return np.ascontiguousarray(v.reshape(shape).transpose(0, 2, 3, 1)).ravel()


def to_logical(name: str, v: np.ndarray, shape: list, cin0_store: int, khwc: bool = False) -> np.ndarray:
    """The inverse of to_store."""
    st = store_shape(name, shape, cin0_store, khwc)
    if st == list(shape):
        return v
    if name == "conv0.w":
        return np.ascontiguousarray(v.reshape(st)[:, :shape[1]]).ravel()
    return np.ascontiguousarray(v.reshape(st).transpose(0, 3, 1, 2)).ravel()


def init_params(specs: list, offsets: dict, flat_len: int, seed: int, cin0_store: int = 3,
                khwc: bool = False) -> np.ndarray:
    """The flat parameter buffer on the host: PyTorch's default Conv2d/Linear
    init (kaiming_uniform_ with a=sqrt(5), i.e. U(+-1/sqrt(fan_in)), for
    weights and biases), BN gamma 1 and beta 0; padding zero.  The values do
    not depend on the storage padding."""
    rng = np.random.default_rng(seed)
    host = np.zeros(flat_len, np.float32)
    for name, shape, init in specs:
        o, n_store = offsets[name]
        n = int(np.prod(shape))
        if init[0] in ("kaiming", "bias"):
            bound = 1.0 / math.sqrt(init[1])
            v = rng.uniform(-bound, bound, n).astype(np.float32)
        else:
            v = np.full(n, init[1], np.float32)
        host[o:o + n_store] = to_store(name, v, shape, cin0_store, khwc)
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
                 weight_decay: float = 5e-4, world: int = 1, comm=None, bucket_bytes: int = 8 << 20,
                 layout: str = "nhwc", keep_acts: bool = False, early_update=None):
        if layout not in ("nhwc", "nchw"):
            raise ValueError(f"layout must be 'nhwc' or 'nchw', got {layout!r}")
        self.layout = layout
        self.cin0 = CIN0_PAD if layout == "nhwc" else 3
        self.khwc = layout == "nhwc"  # conv filters (but the first) stored [Cout][3][3][Cin]
        # channels-last blocks with a pool write only the pooled BN+ReLU values
        # (BN, ReLU and pool in one pass); keep_acts also stores the full-size ones
        self.fuse_pool = layout == "nhwc"
        self.keep_acts = bool(keep_acts) or not self.fuse_pool
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
        specs, self.offsets, self.flat_len = plan_params(self.blocks, self.feat, self.cin0, self.khwc)
        self.param_specs = specs
        self.nparams = sum(int(np.prod(s)) for _, s, _ in specs)
        self.params = self._alloc(self.flat_len * 4)
        self.grads = self._alloc(self.flat_len * 4)
        self.moms = self._alloc(self.flat_len * 4)
        self._h2d(self.params, init_params(specs, self.offsets, self.flat_len, seed, self.cin0, self.khwc))
        # tf32 low parts of the parameters, which the conv kernels read beside the
        # filters (channels-last step only); the SGD step keeps them current
        self.params_lo = self._alloc(self.flat_len * 4) if self.khwc else 0
        if self.params_lo:
            check(self.lib.tpk_tf32_lo(_vp(self.params), _vp(self.params_lo), self.flat_len))
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
        self.x = self._alloc(Bn * 3 * 32 * 32 * 4)  # the batch as it arrives (NCHW)
        self.y = self._alloc(Bn * 4)
        # first conv input: channels-last, zero-padded channels (NCHW: the batch itself)
        self.x0 = self._alloc(Bn * self.cin0 * 32 * 32 * 4) if layout == "nhwc" else self.x
        max_act = Bn * self.cin0 * 32 * 32
        for b in self.blocks:
            n = Bn * b["cout"] * b["H"] * b["W"]
            max_act = max(max_act, n, Bn * b["cin"] * b["H"] * b["W"])
            b["z"] = self._alloc(n * 4)  # conv output (BN input)
            # BN + ReLU output (not kept for fused pooled blocks)
            b["a"] = self._alloc(n * 4) if (self.keep_acts or not b["pool"]) else 0
            if b["pool"]:
                m = n // 4
                b["p"] = self._alloc(m * 4)
                b["idx"] = self._alloc(m * 4)
            b["out"] = b["p"] if b["pool"] else b["a"]
        self.logits = self._alloc(Bn * NUM_CLASSES * 4)
        self.loss_rows = self._alloc(Bn * 4)
        self.loss = self._alloc(4)
        self.dfeat = self._alloc(Bn * self.feat * 4)
        # gradient buffers, used in rotation; channels-last steps run each weight
        # gradient on the auxiliary stream beside the next data gradient, so a
        # buffer is reused only after the weight gradient that read it is done
        self.overlap = layout == "nhwc"
        self.gbuf = [self._alloc(max_act * 4) for _ in range(4 if self.overlap else 2)]

        # ---- optimizer group: every parameter tensor, fused SGD ----
        names = [n for n, _, _ in specs]
        ptr = lambda base: (ctypes.c_void_p * len(names))(*[base + 4 * self.offsets[n][0] for n in names])  # noqa
        numels = (ctypes.c_int64 * len(names))(*[self.offsets[n][1] for n in names])
        # the SGD step also writes the updated tf32 low parts of the conv filters
        # that the tensor-core kernels read in place (all but the first)
        lo_rows = None
        if self.params_lo:
            lo_rows = (ctypes.c_void_p * len(names))(*[
                self.params_lo + 4 * self.offsets[n][0] if (n.startswith("conv") and n.endswith(".w")
                                                            and n != "conv0.w") else None for n in names])
        g = ctypes.c_int64(0)
        check(self.lib.tpk_group_create_lo(len(names), ptr(self.params), ptr(self.grads), ptr(self.moms), None,
                                           lo_rows, numels, ctypes.byref(g)))
        self.group = g.value

        # gradient buckets (contiguous ranges of the flat gradient buffer)
        self._plan_buckets()
        # data-parallel channels-last steps update each bucket's parameters as soon as its
        # gradients are all-reduced and nothing later in the step reads them: one SGD group
        # per bucket, on the side stream, which is then the communicator's (2 GPUs: 2.73 ->
        # 2.70 ms per step).  One GPU keeps a single update at the end unless asked
        # (early_update=True): there the per-bucket launches cost more than they hide
        # (batch 128: 0.927 -> 0.944 ms on the side stream, 1.06 on the auxiliary one)
        if early_update is None:
            early_update = comm is not None
        self.bucket_groups = {}
        if self.overlap and early_update:
            for start, count, key in self.buckets:
                idx = [i for i, n in enumerate(names) if start <= self.offsets[n][0] < start + count]
                pp = (ctypes.c_void_p * len(idx))(*[self.params + 4 * self.offsets[names[i]][0] for i in idx])
                gg = (ctypes.c_void_p * len(idx))(*[self.grads + 4 * self.offsets[names[i]][0] for i in idx])
                mm = (ctypes.c_void_p * len(idx))(*[self.moms + 4 * self.offsets[names[i]][0] for i in idx])
                ll = (ctypes.c_void_p * len(idx))(*[lo_rows[i] for i in idx]) if lo_rows is not None else None
                nn = (ctypes.c_int64 * len(idx))(*[self.offsets[names[i]][1] for i in idx])
                gb = ctypes.c_int64(0)
                check(self.lib.tpk_group_create_lo(len(idx), pp, gg, mm, None, ll, nn, ctypes.byref(gb)))
                self.bucket_groups[key] = gb.value

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

    def p_lo(self, name: str):
        """Device pointer to the tf32 low parts of parameter `name` (None without them)."""
        return _vp(self.params_lo + 4 * self.offsets[name][0]) if self.params_lo else None

    def g(self, name: str) -> int:
        return self.grads + 4 * self.offsets[name][0]

    def _plan_buckets(self) -> None:
        self.buckets = plan_buckets(self.offsets, len(self.blocks), self.flat_len, self.bucket_bytes)
        self.bucket_after = {b[2]: b for b in self.buckets}

    # ---- the step ----------------------------------------------------------------------
    def _forward(self) -> None:
        L = self.lib
        Bn = self.B
        nhwc = self.layout == "nhwc"
        if nhwc:
            check(L.tpk_nchw_to_nhwc(_vp(self.x), _vp(self.x0), Bn, 3, 32, 32, self.cin0))
        x = self.x0
        for li, b in enumerate(self.blocks):
            C, H, W = b["cout"], b["H"], b["W"]
            cin = self.cin0 if li == 0 else b["cin"]
            w, bias = _vp(self.p(f"conv{li}.w")), _vp(self.p(f"conv{li}.b"))
            gam, bet = _vp(self.p(f"bn{li}.g")), _vp(self.p(f"bn{li}.b"))
            stats = (_vp(b["rm"]), _vp(b["rv"]), _vp(b["a"]), _vp(b["mean"]), _vp(b["invstd"]))
            if nhwc:
                check(L.tpk_conv2d_fwd_nhwc_lo(_vp(x), w, self.p_lo(f"conv{li}.w"), bias, _vp(b["z"]), Bn, cin, H,
                                               W, C, 3, 3, 1, 1, self.filter_layout(li)))
                if b["pool"]:
                    check(L.tpk_bn_train_pool_nhwc(_vp(b["z"]), gam, bet, _vp(b["rm"]), _vp(b["rv"]), _vp(b["p"]),
                                                   _vp(b["idx"]), _vp(b["a"]) if b["a"] else None, _vp(b["mean"]),
                                                   _vp(b["invstd"]), Bn, H, W, C, 1e-5, 0.1, 1))
                else:
                    check(L.tpk_bn_train_nhwc(_vp(b["z"]), gam, bet, *stats, Bn * H * W, C, 1e-5, 0.1, 1))
            else:
                check(L.tpk_conv2d_fwd(_vp(x), w, bias, _vp(b["z"]), Bn, cin, H, W, C, 3, 3, 1, 1, 1, 1))
                check(L.tpk_bn_train(_vp(b["z"]), gam, bet, *stats, Bn, C, H * W, 1e-5, 0.1, 1))
                if b["pool"]:
                    check(L.tpk_maxpool_fwd(_vp(b["a"]), _vp(b["p"]), _vp(b["idx"]), Bn, C, H, W, 2, 2, 0))
            x = b["out"]
        # the last block ends at 1x1, where both layouts are [B][512]; the classifier's
        # forward and backward (logits, mean cross-entropy, fc gradients, feature
        # gradient) are one launch
        self.feat_ptr = x
        check(L.tpk_linear_cross_entropy_step(_vp(x), _vp(self.p("fc.w")), _vp(self.p("fc.b")), _vp(self.y),
                                              _vp(self.logits), _vp(self.loss_rows), _vp(self.loss),
                                              _vp(self.dfeat), _vp(self.g("fc.w")), _vp(self.g("fc.b")), Bn,
                                              self.feat, NUM_CLASSES, 1.0 / Bn))

    def _update_bucket(self, key: str) -> None:
        """SGD on the bucket that closes at `key`, once its gradients are final (and
        all-reduced) and nothing later in the step reads its parameters: on the side
        stream, behind the library and auxiliary streams' work so far and the
        bucket's all-reduce; the library stream joins it before the step ends."""
        if key not in self.bucket_groups:
            return
        L = self.lib
        check(L.tp_side_fork())
        try:
            check(L.tpk_sgd_group(self.bucket_groups[key], self.lr, self.momentum, self.wd, 0.0, 0, 1.0 / self.world))
        finally:
            check(L.tp_side_return())

    def _reduce(self, key: str) -> None:
        if self.comm is not None and key in self.bucket_after:
            start, count, _ = self.bucket_after[key]
            self.comm.allreduce_async(self.grads + 4 * start, count)

    def _backward(self) -> None:
        L = self.lib
        Bn = self.B
        # the classifier's gradients were written by the forward's head launch
        self._reduce("fc")
        gout = self.dfeat
        if self.overlap:
            self._update_bucket("fc")  # nothing after the head reads fc.w / fc.b
            self._backward_blocks_overlapped(gout)
            return
        buf = 0
        for li in reversed(range(len(self.blocks))):
            b = self.blocks[li]
            C, H, W = b["cout"], b["H"], b["W"]
            cin = self.cin0 if li == 0 else b["cin"]
            if b["pool"]:
                da = self.gbuf[buf]
                buf ^= 1
                check(L.tpk_maxpool_bwd(_vp(gout), _vp(b["idx"]), _vp(da), Bn, C, H, W, 2, 2, 0))
            else:
                da = gout
            dz = self.gbuf[buf]
            buf ^= 1
            xin = self.x0 if li == 0 else self.blocks[li - 1]["out"]
            w, dw, db = _vp(self.p(f"conv{li}.w")), _vp(self.g(f"conv{li}.w")), _vp(self.g(f"conv{li}.b"))
            bn_args = (_vp(da), _vp(b["z"]), _vp(b["a"]), _vp(self.p(f"bn{li}.g")), _vp(b["mean"]),
                       _vp(b["invstd"]), _vp(dz), _vp(self.g(f"bn{li}.g")), _vp(self.g(f"bn{li}.b")))
            check(L.tpk_bn_backward(*bn_args, Bn, C, H * W))
            check(L.tpk_channel_sum(_vp(dz), Bn, C, H * W, db))
            check(L.tpk_conv2d_wgrad(_vp(dz), _vp(xin), dw, Bn, cin, H, W, C, 3, 3, 1, 1, 1, 1))
            self._reduce(f"blk{li}")
            if li > 0:
                dx = self.gbuf[buf]
                buf ^= 1
                check(L.tpk_conv2d_dgrad(_vp(dz), w, _vp(dx), Bn, cin, H, W, C, 3, 3, 1, 1, 1, 1))
                gout = dx

    def _backward_blocks_overlapped(self, gout: int) -> None:
        """Channels-last block backward: BN backward (pool gradient read in
        place, ReLU mask from z, conv bias gradient from the same pass) and the
        data gradient on the library stream; each weight gradient, and the
        gradient all-reduce of the bucket it closes, on the auxiliary stream
        beside them.  Four gradient buffers in rotation; before the library
        stream writes a buffer that held dz of layer j, it waits for layer j's
        weight gradient (event slot j)."""
        L = self.lib
        Bn = self.B
        holder = [None] * len(self.gbuf)  # layer whose weight gradient reads the buffer's dz
        nxt = [0]

        def take() -> int:
            i = nxt[0]
            nxt[0] = (i + 1) % len(self.gbuf)
            if holder[i] is not None:
                check(L.tp_main_wait(holder[i]))
                holder[i] = None
            return i

        for li in reversed(range(len(self.blocks))):
            b = self.blocks[li]
            C, H, W = b["cout"], b["H"], b["W"]
            cin = self.cin0 if li == 0 else b["cin"]
            iz = take()
            dz = self.gbuf[iz]
            xin = self.x0 if li == 0 else self.blocks[li - 1]["out"]
            w, dw, db = _vp(self.p(f"conv{li}.w")), _vp(self.g(f"conv{li}.w")), _vp(self.g(f"conv{li}.b"))
            # gout is the pooled gradient for pooled blocks (read in place with the pool's indices)
            check(L.tpk_bn_backward_fused_nhwc(_vp(gout), _vp(b["idx"]) if b["pool"] else None, _vp(b["z"]),
                                               _vp(self.p(f"bn{li}.g")), _vp(self.p(f"bn{li}.b")), _vp(b["mean"]),
                                               _vp(b["invstd"]), _vp(dz), _vp(self.g(f"bn{li}.g")),
                                               _vp(self.g(f"bn{li}.b")), db, Bn, H, W, C, 1))
            check(L.tp_aux_fork())
            try:
                check(L.tpk_conv2d_wgrad_nhwc(_vp(dz), _vp(xin), dw, Bn, cin, H, W, C, 3, 3, 1, 1,
                                              self.filter_layout(li)))
                self._reduce(f"blk{li}")
                check(L.tp_aux_record(li))
            finally:
                check(L.tp_aux_return())
            holder[iz] = li
            if li > 0:
                dx = self.gbuf[take()]
                check(L.tpk_conv2d_dgrad_nhwc_lo(_vp(dz), w, self.p_lo(f"conv{li}.w"), _vp(dx), Bn, cin, H, W, C,
                                                 3, 3, 1, 1, self.filter_layout(li)))
                gout = dx
            # the data gradient was the last reader of this block's filters
            self._update_bucket(f"blk{li}")
        check(L.tp_aux_join())

    def _update(self) -> None:
        if self.comm is not None:
            self.comm.wait()
        if self.bucket_groups:  # every bucket was updated during the backward
            check(self.lib.tp_side_join())
        else:
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

    def _logical(self, base: int, name: str) -> np.ndarray:
        o, n = self.offsets[name]
        shape = dict((nm, s) for nm, s, _ in self.param_specs)[name]
        return to_logical(name, self.read(base + 4 * o, n), shape, self.cin0, self.khwc)

    def filter_layout(self, li: int) -> int:
        """filter_layout argument of the channels-last conv entry points for block li."""
        return 1 if self.khwc and li > 0 else 0

    def param_array(self, name: str) -> np.ndarray:
        """Parameter `name` in its logical (reference) layout."""
        return self._logical(self.params, name)

    def grad_array(self, name: str) -> np.ndarray:
        """Gradient of `name` from the last step, logical layout."""
        return self._logical(self.grads, name)

    def activation(self, ptr: int, C: int, H: int, W: int, dtype=np.float32) -> np.ndarray:
        """A [B][C][H][W] activation (or int32 pool index) read back as NCHW."""
        n = self.B * C * H * W
        out = np.zeros(n, dtype)
        check(self.lib.tp_memcpy_d2h(out.ctypes.data_as(ctypes.c_void_p), _vp(ptr), out.nbytes))
        if self.layout == "nhwc":
            return np.ascontiguousarray(out.reshape(self.B, H, W, C).transpose(0, 3, 1, 2))
        return out.reshape(self.B, C, H, W)

    def close(self) -> None:
        if self.graph is not None:
            self.lib.tp_graph_destroy(self.graph)
            self.graph = None
        self.lib.tpk_group_destroy(self.group)
        for g in self.bucket_groups.values():
            self.lib.tpk_group_destroy(g)
        self.bucket_groups = {}
        for p in self._allocs:
            self.lib.tp_free(_vp(p))
        self._allocs = []

    # algorithmic work of one step at this batch (for the roofline)
    def step_roofline_ms(self, tensor_tflops: float, cuda_tflops: float, hbm_gbs: float) -> dict:
        """Lower bound of the step's time from its algorithmic work: the
        tensor-core convolutions (3xTF32 flops of fwd + data gradient + weight
        gradient) at `tensor_tflops`, the first layer (CUDA cores, 3 real input
        channels) at `cuda_tflops`, and the HBM-bound passes at `hbm_gbs` --
        BatchNorm statistics / apply (+ pool) / backward (two passes, the pooled
        gradient and argmax read in place) and the fused SGD."""
        tensor = cuda = hbm = 0.0
        for li, b in enumerate(self.blocks):
            macs = self.B * b["cout"] * b["H"] * b["W"] * (3 if li == 0 else b["cin"]) * 9
            if li == 0:
                cuda += 2 * macs * 2 / (cuda_tflops * 1e12)
            else:
                tensor += 2 * macs * 3 / (tensor_tflops * 1e12)
            e = 4.0 * self.B * b["cout"] * b["H"] * b["W"]  # bytes of one activation tensor
            if b["pool"]:
                hbm += e + e * 1.5  # statistics; apply + ReLU + pool (read z, write pooled value and index)
                hbm += 1.5 * e + 2.5 * e  # backward: sums (z, pooled g, index); apply (same + write dz)
            else:
                hbm += e + 2 * e  # statistics; apply + ReLU
                hbm += 2 * e + 3 * e  # backward: sums (z, g); apply (z, g, write dz)
        hbm += 24.0 * self.nparams  # SGD: param, grad, momentum read; param, momentum, tf32 low part written
        hbm_s = hbm / (hbm_gbs * 1e9)
        total = tensor + cuda + hbm_s
        return {"min_ms": total * 1e3, "tensor_ms": tensor * 1e3, "cuda_core_ms": cuda * 1e3, "hbm_ms": hbm_s * 1e3,
                "hbm_bytes": hbm}

    def step_flops(self) -> float:
        f = 0.0
        for li, b in enumerate(self.blocks):
            macs = self.B * b["cout"] * b["H"] * b["W"] * b["cin"] * 9
            f += 2 * macs * (3 if li > 0 else 2)  # fwd + wgrad (+ dgrad except layer 1)
        f += 2 * self.B * self.feat * NUM_CLASSES * 3
        return f
