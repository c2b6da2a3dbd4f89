"""A few training steps of a CNN through a torch API, written once and run by
the drop-in tests in a subprocess on one of three back ends:

  oracle  the unmodified reference ``torch`` package (from baseline/_ref or
          the reference checkout) over the CPU oracle runtime, with
          tpcuda.patches applied;
  cuda    the same package and patches over the CUDA runtime;
  torch   real PyTorch on the CPU, as an independent cross-check of the
          training semantics (PyTorch's rules for max-pool, BatchNorm and
          LayerNorm backward, which the patches implement).

  python dropin_train.py <backend> <model> <steps> <out.npz> [optimizer]

Every back end starts from the same numpy-seeded weights (loaded with
load_state_dict) and batch, and writes the per-step losses, the last step's
parameter gradients (and the first step's), the final parameters to out.npz,
plus the runtime's allocated bytes after each step (the lifetime check).
"""
import gc
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def reference_path():
    for p in (os.path.join(ROOT, "baseline", "_ref"), "/root/reference/python"):
        if os.path.isdir(os.path.join(p, "torch")):
            return p
    return None


def main():
    backend, model_name, steps, out = sys.argv[1], sys.argv[2], int(sys.argv[3]), sys.argv[4]
    opt_name = sys.argv[5] if len(sys.argv) > 5 else "sgd"
    rt = None
    if backend in ("oracle", "cuda"):
        sys.path[:0] = [os.path.join(ROOT, "torch-pyodide_b200"), os.path.join(ROOT, "oracle")]
        from tpcuda import patches, shim
        if backend == "oracle":
            from oracle_runtime import OracleRuntime
            rt = OracleRuntime()
        else:
            from tpcuda import CudaRuntime
            rt = CudaRuntime(0)
        shim.install(rt)
        sys.path.insert(0, reference_path())
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    if rt is not None:
        assert "site-packages" not in torch.__file__ or "_ref" in torch.__file__, torch.__file__
        patches.apply()

    def conv_bn(cin, cout):
        return [nn.Conv2d(cin, cout, 3, padding=1), nn.BatchNorm2d(cout), nn.ReLU()]

    if model_name == "tiny":  # the Tiny CNN training config (batch 64, 1x28x28)
        layers = [nn.Conv2d(1, 8, 3, padding=1), nn.ReLU(), nn.MaxPool2d(2), nn.Conv2d(8, 16, 3, padding=1),
                  nn.ReLU(), nn.MaxPool2d(2), nn.Flatten(), nn.Linear(784, 10)]
        B, shape = 64, (1, 28, 28)
    elif model_name == "vgg":  # VGG-11-BN (CIFAR head), the data-parallel config's network
        cfg = [64, "M", 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"]
        layers, cin = [], 3
        for v in cfg:
            if v == "M":
                layers.append(nn.MaxPool2d(2))
            else:
                layers += conv_bn(cin, v)
                cin = v
        layers += [nn.Flatten(), nn.Linear(512, 10)]
        B, shape = 8, (3, 32, 32)
    else:  # a small CNN with every rebound op: conv, BN, ReLU, max-pool, linear, LayerNorm
        layers = conv_bn(3, 8) + [nn.MaxPool2d(2)] + conv_bn(8, 16) + [nn.MaxPool2d(2), nn.Flatten(),
                                                                        nn.Linear(256, 10), nn.LayerNorm(10)]
        B, shape = 4, (3, 16, 16)
    model = nn.Sequential(*layers)
    model.train()

    rng = np.random.default_rng(1234)
    named = dict(model.named_parameters())
    names = list(named)
    sd = {}
    for n in names:
        shp = tuple(named[n].shape)
        if n.endswith("weight") and len(shp) > 1:
            fan_in = int(np.prod(shp[1:]))
            arr = rng.standard_normal(shp) * np.sqrt(2.0 / fan_in)
        elif n.endswith("weight"):  # BatchNorm / LayerNorm gamma
            arr = 1.0 + 0.1 * rng.standard_normal(shp)
        else:
            arr = 0.1 * rng.standard_normal(shp)
        sd[n] = torch.tensor(np.asarray(arr, np.float32))
    model.load_state_dict(sd, strict=False)
    x = torch.tensor(rng.standard_normal((B,) + shape).astype(np.float32))
    y = torch.tensor(rng.integers(0, 10, B).astype(np.int64), dtype=torch.int64)
    params = [p for _, p in model.named_parameters()]
    if opt_name == "adam":
        opt = torch.optim.Adam(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8)
    elif opt_name == "adamw":
        opt = torch.optim.AdamW(params, lr=1e-3, weight_decay=0.01)
    else:  # momentum and weight decay of the data-parallel config; a smaller lr on
        # the deep net keeps 3 steps of batch 8 away from chaotic ReLU / max-pool flips,
        # and from fitting the 8 images at once (at lr 0.005 the loss falls 2.84 -> 0.004
        # in one step, after which the first layer's gradient is a sum that cancels to
        # ~1% of its terms, so the comparison would measure rounding, not the kernels)
        opt = torch.optim.SGD(params, lr=5e-4 if model_name == "vgg" else 0.05, momentum=0.9, weight_decay=5e-4)

    def arr(t):
        return np.asarray(t.detach().tolist() if hasattr(t, "detach") else t.tolist(), np.float32)

    losses, live = [], []
    grads, first_grads = {}, {}
    for _ in range(steps):
        opt.zero_grad()
        loss = F.cross_entropy(model(x), y)
        loss.backward()
        losses.append(float(loss.item()))
        grads = {n: arr(p.grad) for n, p in zip(names, params)}
        if not first_grads:
            first_grads.update(grads)
        opt.step()
        del loss
        gc.collect()
        if rt is not None:
            live.append(rt.memoryAllocated())
    res = {"losses": np.asarray(losses), "live": np.asarray(live, np.int64)}
    ckpt = os.environ.get("DROPIN_CKPT")
    if ckpt:  # the trained state dict through torch.save / torch.load (PyTorch's zip format)
        torch.save(model.state_dict(), ckpt)
        back = torch.load(ckpt, weights_only=False)
        mine = model.state_dict(keep_vars=True) if rt is not None else model.state_dict()
        same = set(back) == set(mine) and all(
            np.array_equal(np.asarray(back[k].tolist(), np.float64), np.asarray(mine[k].tolist(), np.float64))
            for k in mine)
        res["ckpt_roundtrip_exact"] = np.asarray(same)
        for k, v in mine.items():
            res["state:" + k] = np.asarray(v.tolist(), np.float64)
    for n, p in zip(names, params):
        res["param:" + n] = arr(p)
        res["grad:" + n] = grads[n]
        res["grad0:" + n] = first_grads[n]
    np.savez(out, **res)


if __name__ == "__main__":
    main()
