"""Generate the golden fixtures in tests/golden/ (run in this repository's dev
container, where the reference checkout is mounted; the GPU tests only read
the JSON files this writes).

Two kinds of fixture:

1. ``reference_examples.json`` -- the recorded outputs of the reference's own
   playground examples (runtime/playground/example-results.json) next to the
   output of the same example script (runtime/playground/public/examples/*.py)
   run by the unmodified reference ``torch`` package on the CPU oracle through
   the drop-in shim.  Only examples whose recorded output is deterministic given
   the script and whose script is unchanged since the recording are kept.
   tests/test_oracle_golden.py pins the oracle against the recorded values.

2. ``traces/<name>.json`` -- the exact stream of runtime calls the reference
   package issues for a script (method, arguments, returned handles) and every
   ``toList`` result, recorded on the oracle.  tests/test_gpu_replay.py replays
   a trace on the CUDA runtime and compares each ``toList`` result, which checks
   the CUDA backend against the oracle on the reference's own op stream without
   needing the reference package at test time.

Usage: python tests/golden/make_golden.py [--reference /root/reference]
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# (example id in example-results.json, script file, keys compared)
EXAMPLES = [
    ("rand_tensor", "rand_tensor.py", ["shape", "values"]),
    ("randn_tensor", "randn_tensor.py", ["shape", "values"]),
    ("tensor_basics", "tensor_basics.py", ["shape", "values", "sum", "mean"]),
    ("matmul_relu", "matmul_relu.py", ["shape", "values", "sum"]),
    ("reshape_transpose", "reshape_transpose.py", ["transpose", "reshape"]),
    ("autograd_basic", "autograd_basic.py", ["loss", "a.grad", "b.grad"]),
    ("autograd_conv2d", "autograd_conv2d_backward.py",
     ["output_shape", "loss", "weight_grad_shape", "weight_grad_sum", "bias_grad", "input_grad_shape"]),
]

# Scripts whose runtime-call stream is recorded as a replay trace.  The
# example scripts above run in one session (as the playground does, so the
# seed counter advances the same way), then the Tiny-CNN training config.
TINY_CNN = r'''
import json
import torch
import torch.nn as nn
import torch.nn.functional as F
torch.manual_seed(0)
class TinyCNN(nn.Module):
    def __init__(self):
        super().__init__()
        self.conv1 = nn.Conv2d(1, 8, 3, padding=1)
        self.conv2 = nn.Conv2d(8, 16, 3, padding=1)
        self.fc = nn.Linear(784, 10)
    def forward(self, x):
        x = F.max_pool2d(F.relu(self.conv1(x)), 2)
        x = F.max_pool2d(F.relu(self.conv2(x)), 2)
        x = x.flatten(1)
        return self.fc(x)
model = TinyCNN()
opt = torch.optim.Adam(model.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8)
x = torch.randn((BATCH, 1, 28, 28))
y = torch.tensor([float(i % 10) for i in range(BATCH)])
losses = []
for step in range(STEPS):
    opt.zero_grad()
    loss = F.cross_entropy(model(x), y)
    loss.backward()
    opt.step()
    losses.append(loss.item())
print(json.dumps({"losses": losses, "fc_weight_sum": model.fc.weight.sum().item()}))
'''


def _child(reference: str, mode: str, out_path: str) -> None:
    """Runs in a fresh interpreter whose `torch` is the reference package."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "torch-pyodide_b200"))
    from oracle_runtime import OracleRuntime
    from tpcuda import shim

    class Recorder(OracleRuntime):
        """OracleRuntime that logs every call; ids start at 1e9 so a replay can
        tell tensor ids from shape integers."""

        def __init__(self):
            super().__init__()
            self._next = 1_000_000_000
            self.trace = []
            self._depth = [0]

        def __getattribute__(self, name):
            attr = object.__getattribute__(self, name)
            if name.startswith("_") or not callable(attr) or name in ("array", "trace"):
                return attr
            trace = object.__getattribute__(self, "trace")
            depth = object.__getattribute__(self, "_depth")

            def wrapped(*args):
                depth[0] += 1
                try:
                    res = attr(*args)
                finally:
                    depth[0] -= 1
                if depth[0] == 0:  # record only the calls the reference package made
                    rec = {"m": name, "a": list(args), "r": res}
                    trace.append(json.loads(json.dumps(rec, default=float)))
                return res
            return wrapped

    rt = Recorder()
    shim.install(rt)
    sys.path.insert(0, os.path.join(reference, "python"))
    import torch  # noqa: F401  (the reference package)

    ex_dir = os.path.join(reference, "runtime", "playground", "public", "examples")
    results = {}
    traces = {}
    if mode == "examples":
        for ex_id, script, _keys in EXAMPLES:
            start = len(rt.trace)
            seed0 = object.__getattribute__(rt, "_seed")
            buf = io.StringIO()
            with contextlib.redirect_stdout(buf):
                exec(compile(open(os.path.join(ex_dir, script)).read(), script, "exec"), {"__name__": "__main__"})
            results[ex_id] = json.loads(buf.getvalue())
            # the playground runs examples in one page session, so the seed
            # counter carries over; a trace starts by restoring it
            traces[ex_id] = [{"m": "setSeed", "a": [seed0], "r": None}] + rt.trace[start:]
    else:
        batch, steps = (64, 10) if mode == "tiny_cnn" else (8, 2)
        src = TINY_CNN.replace("BATCH", str(batch)).replace("STEPS", str(steps))
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            exec(compile(src, "tiny_cnn", "exec"), {"__name__": "__main__"})
        results[mode] = json.loads(buf.getvalue())
        traces[mode] = rt.trace
    json.dump({"results": results, "traces": traces}, open(out_path, "w"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--child", default=None)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    if args.child:
        _child(args.reference, args.child, args.out)
        return

    recorded = {e["id"]: e for e in json.load(open(os.path.join(
        args.reference, "runtime", "playground", "example-results.json")))}
    os.makedirs(os.path.join(HERE, "traces"), exist_ok=True)
    tmp = os.path.join(HERE, "_tmp.json")
    golden = {}
    for mode in ("examples", "tiny_cnn", "tiny_cnn_small"):
        subprocess.run([sys.executable, __file__, "--reference", args.reference, "--child", mode, "--out", tmp],
                       check=True, cwd=ROOT)
        data = json.load(open(tmp))
        for name, trace in data["traces"].items():
            json.dump({"name": name, "result": data["results"][name], "calls": trace},
                      open(os.path.join(HERE, "traces", f"{name}.json"), "w"), separators=(",", ":"))
        if mode == "examples":
            for ex_id, script, keys in EXAMPLES:
                rec = recorded[ex_id]
                assert rec["success"], ex_id
                rec_out = json.loads(rec["output"])
                golden[ex_id] = {"script": script, "keys": keys,
                                 "recorded": {k: rec_out[k] for k in keys},
                                 "oracle": {k: data["results"][ex_id][k] for k in keys}}
    os.remove(tmp)
    json.dump(golden, open(os.path.join(HERE, "reference_examples.json"), "w"), indent=1)
    print("wrote", len(golden), "examples and traces to", HERE)


if __name__ == "__main__":
    main()
