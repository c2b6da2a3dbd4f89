"""VGG-11-BN training step composed from the CPU oracle's op restatements.

TEST INFRASTRUCTURE ONLY: the checker for tpcuda.vgg (tests/test_gpu_vgg.py)
and the CPU baseline of bench.py.  Each op is the oracle restatement of the
reference shader (conv.wgsl, conv_backward.wgsl, max_pool2d.wgsl, ...) or of
the intended training semantics the reference composes in Python
(tensor_nn_ops.py:92-254 BN training; PyTorch's BN / max-pool backward rules).
"""
from __future__ import annotations

import numpy as np


def oracle_step(orc, model, params, x, y, bn_stats, lr, mom, wd):
    """One step of the same network on the oracle; returns (loss, new params, running stats)."""
    loss, G, P, stats = _forward_backward(orc, model, params, x, y, bn_stats)
    names = list(params)
    moms = [_tensor(orc, np.zeros(int(np.prod(params[n][1])))) for n in names]
    orc.sgdStepMulti([P[n] for n in names], [G[n] for n in names], moms, lr, mom, wd, 0.0, False)
    new = {n: np.asarray(orc.toList(P[n]), np.float32) for n in names}
    return loss, new, stats


def oracle_grads(orc, model, params, x, y, bn_stats):
    """Forward and backward of the same network on the oracle (free running);
    returns (loss, {parameter name: gradient array})."""
    loss, G, _, _ = _forward_backward(orc, model, params, x, y, bn_stats)
    return loss, {n: np.asarray(orc.toList(G[n]), np.float32) for n in params}


def _tensor(orc, a, shape=None):
    a = np.ascontiguousarray(a, np.float32)
    return orc.tensorFromData(a.ravel().tolist(), list(shape or a.shape), "float32")["id"]


def _forward_backward(orc, model, params, x, y, bn_stats):
    def T(a, shape=None):
        a = np.ascontiguousarray(a, np.float32)
        return orc.tensorFromData(a.ravel().tolist(), list(shape or a.shape), "float32")["id"]

    P = {k: T(v, s) for k, (v, s) in params.items()}
    stat_ids = [(T(rm), T(rv)) for rm, rv in bn_stats]
    loss, G = _forward_backward_ids(orc, model, P, T(x), T(y), stat_ids, x.shape[0])
    stats = [(np.asarray(orc.toList(rm), np.float32), np.asarray(orc.toList(rv), np.float32)) for rm, rv in stat_ids]
    return loss, G, P, stats


def _forward_backward_ids(orc, model, P, xin, yt, stat_ids, B):
    """Forward and backward over oracle tensors already registered: P maps
    parameter names to ids, stat_ids holds each block's (running mean, running
    var) ids, updated in place by the BN forward.  Returns (loss, {name: grad id})."""
    saved = []
    h = xin
    for li, b in enumerate(model.blocks):
        rm, rv = stat_ids[li]
        z = orc.conv2d(h, P[f"conv{li}.w"], orc.toList(P[f"conv{li}.b"]), [1], [1], [1], 1)["id"]
        yb, mean, inv = [r["id"] for r in orc.batchNormTrain(z, P[f"bn{li}.g"], P[f"bn{li}.b"], rm, rv, 1e-5, 0.1)]
        a = orc.relu(yb)["id"]
        rec = {"x": h, "z": z, "a": a, "mean": mean, "inv": inv}
        if b["pool"]:
            pm, idx = [r["id"] for r in orc.maxPool2dWithIndices(a, [2], [2], [0], [1])]
            rec["idx"] = idx
            h = pm
        else:
            h = a
        saved.append(rec)
    feat = orc.reshape(h, [B, 512])["id"]
    logits = orc.add(orc.matmul(feat, orc.transpose2d(P["fc.w"])["id"])["id"], P["fc.b"])["id"]
    loss = orc.toList(orc.mean(orc.crossEntropy(logits, yt)["id"])["id"])[0]
    one = orc.full([1], 1.0, "float32")["id"]
    dlog = orc.crossEntropyBackward(one, logits, yt, "mean")["id"]
    G = {"fc.w": orc.matmul(orc.transpose2d(dlog)["id"], feat)["id"], "fc.b": orc.sumDim(dlog, 0, False)["id"]}
    g = orc.reshape(orc.matmul(dlog, P["fc.w"])["id"], [B, 512, 1, 1])["id"]
    zero = orc.full([1], 0.0, "float32")["id"]
    for li in reversed(range(len(model.blocks))):
        b, rec = model.blocks[li], saved[li]
        C, H, W = b["cout"], b["H"], b["W"]
        ashape = [B, C, H, W]
        if b["pool"]:
            g = orc.maxPool2dBackward(g, rec["idx"], ashape, [2], [2], [0], [1])["id"]
        g = orc.mul(g, orc.gt(rec["a"], zero)["id"])["id"]
        dz, dgm, dbt = [r["id"] for r in orc.batchNormBackward(g, rec["z"], P[f"bn{li}.g"], rec["mean"], rec["inv"])]
        G[f"bn{li}.g"], G[f"bn{li}.b"] = dgm, dbt
        G[f"conv{li}.b"] = orc.conv2dBiasBackward(dz, C, ashape)["id"]
        xshape = [B, b["cin"], H, W]
        G[f"conv{li}.w"] = orc.conv2dWeightBackward(dz, rec["x"], [C, b["cin"], 3, 3], ashape, xshape, [1], [1])["id"]
        if li > 0:
            g = orc.conv2dInputBackward(dz, P[f"conv{li}.w"], xshape, ashape, [1], [1])["id"]
    return loss, G


class OracleTrainer:
    """The whole training step on the oracle with the model resident in the
    oracle runtime (parameters, momentum buffers and BN running statistics are
    registered once and updated in place, as a runtime that owns device memory
    keeps them): per step the batch is uploaded, forward + backward run, and one
    multi-tensor SGD step (momentum, weight decay) updates every parameter.
    Everything a step creates is released at its end."""

    def __init__(self, orc, model, params, bn_stats, lr, mom, wd):
        self.orc, self.model, self.lr, self.mom, self.wd = orc, model, lr, mom, wd
        self.names = list(params)
        self.P = {k: orc.tensorFromData(np.ascontiguousarray(v, np.float32).ravel(), list(s), "float32")["id"]
                  for k, (v, s) in params.items()}
        self.M = {k: orc.zeros(list(s), "float32")["id"] for k, (_, s) in params.items()}
        self.stats = [(orc.tensorFromData(np.asarray(rm, np.float32), [rm.size], "float32")["id"],
                       orc.tensorFromData(np.asarray(rv, np.float32), [rv.size], "float32")["id"])
                      for rm, rv in bn_stats]

    def step(self, x: np.ndarray, y: np.ndarray) -> float:
        orc = self.orc
        first = orc._next
        xin = orc.tensorFromData(np.ascontiguousarray(x, np.float32).ravel(), list(x.shape), "float32")["id"]
        yt = orc.tensorFromData(np.ascontiguousarray(y, np.float32).ravel(), [y.size], "float32")["id"]
        loss, G = _forward_backward_ids(orc, self.model, self.P, xin, yt, self.stats, x.shape[0])
        orc.sgdStepMulti([self.P[n] for n in self.names], [G[n] for n in self.names],
                         [self.M[n] for n in self.names], self.lr, self.mom, self.wd, 0.0, False)
        for tid in [t for t in orc._t if t >= first]:
            orc.destroy(tid)
        return loss


def oracle_backward(orc, model, params, x, y, saved, logits):
    """The backward of the same step on the oracle, driven by forward state
    taken from the device run (teacher forcing): per block the conv output z,
    the BN+ReLU output a, the pool argmax indices, the batch mean / inv_std,
    and the logits.  ReLU masks and max-pool routing are then the device's own
    decisions, so near-ties cannot send a gradient down a different path; what
    remains to compare is the arithmetic of every backward op.
    Returns {parameter name: gradient array}."""
    B = x.shape[0]

    def T(a, shape=None):
        a = np.ascontiguousarray(a, np.float32)
        return orc.tensorFromData(a.ravel().tolist(), list(shape or a.shape), "float32")["id"]

    P = {k: T(v, s) for k, (v, s) in params.items()}
    yt = T(y)
    lg = T(logits, [B, 10])
    last = model.blocks[-1]
    feat = T(saved[-1]["p"], [B, 512])
    one = T(np.ones(1))
    dlog = orc.crossEntropyBackward(one, lg, yt, "mean")["id"]
    G = {"fc.w": orc.matmul(orc.transpose2d(dlog)["id"], feat)["id"], "fc.b": orc.sumDim(dlog, 0, False)["id"]}
    g = orc.reshape(orc.matmul(dlog, P["fc.w"])["id"], [B, 512, 1, 1])["id"]
    zero = T(np.zeros(1))
    for li in reversed(range(len(model.blocks))):
        b, sv = model.blocks[li], saved[li]
        C, H, W = b["cout"], b["H"], b["W"]
        ashape = [B, C, H, W]
        a = T(sv["a"], ashape)
        z = T(sv["z"], ashape)
        if b["pool"]:
            idx = T(sv["idx"].astype(np.float32), [B, C, H // 2, W // 2])
            g = orc.maxPool2dBackward(g, idx, ashape, [2], [2], [0], [1])["id"]
        g = orc.mul(g, orc.gt(a, zero)["id"])["id"]
        dz, dgm, dbt = [r["id"] for r in orc.batchNormBackward(g, z, P[f"bn{li}.g"], T(sv["mean"]),
                                                                T(sv["invstd"]))]
        G[f"bn{li}.g"], G[f"bn{li}.b"] = dgm, dbt
        G[f"conv{li}.b"] = orc.conv2dBiasBackward(dz, C, ashape)["id"]
        xshape = [B, b["cin"], H, W]
        xin = T(x) if li == 0 else T(saved[li - 1]["out"], xshape)
        G[f"conv{li}.w"] = orc.conv2dWeightBackward(dz, xin, [C, b["cin"], 3, 3], ashape, xshape, [1], [1])["id"]
        if li > 0:
            g = orc.conv2dInputBackward(dz, P[f"conv{li}.w"], xshape, ashape, [1], [1])["id"]
    return {n: np.asarray(orc.toList(G[n]), np.float32) for n in params}
