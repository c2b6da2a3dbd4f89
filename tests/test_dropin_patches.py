"""tpcuda.patches on the CPU: the unmodified reference package, patched, over
the oracle runtime.

* Training semantics: a small CNN (conv, BatchNorm, ReLU, max-pool, linear,
  LayerNorm) and the Tiny CNN config train 3 steps through the patched
  reference package and through real PyTorch (a separate process, as an
  independent cross-check of the rules the patches implement: PyTorch's
  max-pool, BatchNorm and LayerNorm backward).  Losses, first-step gradients
  and final parameters agree to 1e-4 of their scale.
* Lifetime (D7): the runtime's allocated bytes stay flat across steps.
* The fused optimizer groups give the same bits as the reference's own
  per-parameter loops (RMSprop, Adagrad, Adamax, NAdam, RAdam, SGD, Adam, AdamW).
* Checkpoints: torch.save through the byte entries writes the same archive as
  the reference's tolist() path, real PyTorch loads it, and torch.load returns
  the same values.
* Every runtime method the patched reference calls exists on CudaRuntime.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
from dropin_train import reference_path  # noqa: E402

REF = reference_path()
pytestmark = pytest.mark.skipif(REF is None, reason="reference package not installed (baseline/_ref)")
ENV = dict(os.environ, OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "8"))


def run_train(backend, model, steps, out, opt="sgd", env=None):
    r = subprocess.run([sys.executable, os.path.join(HERE, "dropin_train.py"), backend, model, str(steps), str(out),
                        opt], capture_output=True, text=True, timeout=900, env=env or ENV)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return np.load(out)


# Conv biases feeding a BatchNorm have a mathematically zero gradient: both
# sides hold rounding noise there, which Adam-type steps (m / sqrt(v)) turn
# into full-size updates.  Such parameters (first-step gradient below 1e-6 of
# the largest) are left out of the comparison; the rest is compared at `rel`.
def compare(a, b, rel=1e-4, floor=1e-6):
    gmax = max(float(np.max(np.abs(b[k]))) for k in b.files if k.startswith("grad0:"))
    noise = {k.split(":", 1)[1] for k in b.files if k.startswith("grad0:") and
             float(np.max(np.abs(b[k]))) < 1e-6 * gmax}
    worst = {}
    for k in a.files:
        if k in ("live",) or (":" in k and k.split(":", 1)[1] in noise):
            continue
        x, y = a[k].astype(np.float64), b[k].astype(np.float64)
        assert x.shape == y.shape, k
        scale = max(float(np.max(np.abs(y))) if y.size else 0.0, floor / rel)
        err = float(np.max(np.abs(x - y))) if y.size else 0.0
        worst[k] = err / scale
        assert err <= rel * scale, (k, err, scale)
    return worst


@pytest.mark.parametrize("model,opt", [("cnn", "sgd"), ("cnn", "adamw"), ("tiny", "adam")])
def test_patched_reference_trains_like_pytorch(tmp_path, model, opt):
    a = run_train("oracle", model, 3, tmp_path / "o.npz", opt)
    b = run_train("torch", model, 3, tmp_path / "t.npz", opt)
    compare(a, b)
    live = a["live"]
    assert len(live) == 3 and live[0] == live[-1] > 0, live  # no growth across steps (D7)


OPT_SCRIPT = r"""
import sys, json
import numpy as np
sys.path[:0] = [{pkg!r}, {orc!r}]
from tpcuda import shim, patches
from oracle_runtime import OracleRuntime
rt = OracleRuntime(); shim.install(rt)
sys.path.insert(0, {ref!r})
import torch, torch.nn as nn, torch.nn.functional as F
if {patched}:
    patches.apply()
rng = np.random.default_rng(3)
model = nn.Sequential(nn.Linear(20, 16), nn.ReLU(), nn.Linear(16, 5))
sd = {{n: torch.tensor((rng.standard_normal(tuple(p.shape)) * 0.3).astype(np.float32).tolist())
      for n, p in model.named_parameters()}}
model.load_state_dict(sd, strict=False)
x = torch.tensor(rng.standard_normal((8, 20)).astype(np.float32).tolist())
y = torch.tensor(rng.integers(0, 5, 8).tolist(), dtype=torch.int64)
opts = dict(rmsprop=lambda p: torch.optim.RMSprop(p, lr=0.01, momentum=0.9, weight_decay=0.01),
            rmsprop0=lambda p: torch.optim.RMSprop(p, lr=0.01),
            adagrad=lambda p: torch.optim.Adagrad(p, lr=0.05, lr_decay=0.01, weight_decay=0.01),
            adamax=lambda p: torch.optim.Adamax(p, lr=0.01, weight_decay=0.01),
            nadam=lambda p: torch.optim.NAdam(p, lr=0.01, weight_decay=0.01),
            radam=lambda p: torch.optim.RAdam(p, lr=0.01),
            sgd=lambda p: torch.optim.SGD(p, lr=0.05, momentum=0.9, weight_decay=5e-4, nesterov=True),
            adam=lambda p: torch.optim.Adam(p, lr=0.01, weight_decay=0.01),
            adamw=lambda p: torch.optim.AdamW(p, lr=0.01, weight_decay=0.01))
opt = opts[{name!r}](list(model.parameters()))
for _ in range(7):
    opt.zero_grad()
    F.cross_entropy(model(x), y).backward()
    opt.step()
print(json.dumps([[float(v) for v in np.asarray(p.tolist(), np.float32).ravel()] for p in model.parameters()]))
"""


@pytest.mark.parametrize("name", ["rmsprop", "rmsprop0", "adagrad", "adamax", "nadam", "radam", "sgd", "adam",
                                  "adamw"])
def test_fused_optimizer_groups_equal_reference_loops(name):
    outs = []
    for patched in (False, True):
        code = OPT_SCRIPT.format(pkg=os.path.join(ROOT, "torch-pyodide_b200"), orc=os.path.join(ROOT, "oracle"),
                                 ref=REF, patched=patched, name=name)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, env=ENV)
        assert r.returncode == 0, r.stderr[-3000:]
        outs.append(json.loads(r.stdout.strip().splitlines()[-1]))
    assert outs[0] == outs[1]  # bit for bit: same kernels' arithmetic, same host-side scalars


CKPT_SCRIPT = r"""
import sys, io, json, os
import numpy as np
sys.path[:0] = [{pkg!r}, {orc!r}]
from tpcuda import shim, patches
from oracle_runtime import OracleRuntime
rt = OracleRuntime(); shim.install(rt)
sys.path.insert(0, {ref!r})
import torch, torch.nn as nn
torch.manual_seed(0)
model = nn.Sequential(nn.Conv2d(3, 4, 3), nn.BatchNorm2d(4), nn.Flatten(), nn.Linear(4 * 6 * 6, 5))
model.train()
model(torch.randn(2, 3, 8, 8))  # running stats and num_batches_tracked move
raw = io.BytesIO(); torch.save(model.state_dict(), raw)
patches.apply()
fast = io.BytesIO(); torch.save(model.state_dict(), fast)
open({path!r}, "wb").write(fast.getvalue())
back = torch.load(io.BytesIO(fast.getvalue()))
vals = {{k: (np.asarray(v.tolist(), np.float64).ravel().tolist(), str(v.dtype)) for k, v in back.items()}}
orig = {{k: (np.asarray(v.tolist(), np.float64).ravel().tolist(), str(v.dtype))
        for k, v in model.state_dict(keep_vars=True).items()}}
print(json.dumps({{"same_bytes": raw.getvalue() == fast.getvalue(), "equal": vals == orig, "vals": vals}}))
"""


def test_checkpoint_bytes_identical_and_loadable_by_pytorch(tmp_path):
    path = tmp_path / "sd.pt"
    code = CKPT_SCRIPT.format(pkg=os.path.join(ROOT, "torch-pyodide_b200"), orc=os.path.join(ROOT, "oracle"),
                              ref=REF, path=str(path))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, env=ENV)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["same_bytes"] and res["equal"]
    # real PyTorch reads the archive (PyTorch's zipfile format) to the same values
    chk = ("import json, torch; sd = torch.load(%r, weights_only=False); "
           "print(json.dumps({k: v.double().flatten().tolist() for k, v in sd.items()}))" % str(path))
    r2 = subprocess.run([sys.executable, "-c", chk], capture_output=True, text=True, timeout=300)
    assert r2.returncode == 0, r2.stderr[-3000:]
    real = json.loads(r2.stdout.strip().splitlines()[-1])
    assert set(real) == set(res["vals"])
    for k, v in real.items():
        assert v == res["vals"][k][0], k


REC_SCRIPT = r"""
import sys, json
sys.path[:0] = [{pkg!r}, {orc!r}, {here!r}]
from tpcuda import shim
from oracle_runtime import OracleRuntime
called = set()
class Rec:
    def __init__(self, rt): self._rt = rt
    def __getattr__(self, n):
        called.add(n)
        return getattr(self._rt, n)
import tpcuda.shim as S
orig = S.install
S.install = lambda rt: orig(Rec(rt))
import dropin_train
sys.argv = ["x", "oracle", {model!r}, "2", {out!r}, {opt!r}]
dropin_train.main()
print(json.dumps(sorted(called)))
"""


@pytest.mark.parametrize("model,opt", [("cnn", "adamw"), ("tiny", "adam")])
def test_patched_reference_calls_only_methods_cuda_runtime_has(tmp_path, model, opt):
    from tpcuda.runtime import CudaRuntime
    code = REC_SCRIPT.format(pkg=os.path.join(ROOT, "torch-pyodide_b200"), orc=os.path.join(ROOT, "oracle"),
                             here=HERE, model=model, out=str(tmp_path / "r.npz"), opt=opt)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, env=ENV)
    assert r.returncode == 0, r.stderr[-3000:]
    called = json.loads(r.stdout.strip().splitlines()[-1])
    missing = [m for m in called if not callable(getattr(CudaRuntime, m, None))]
    assert not missing, missing
    assert {"maxPool2dWithIndices", "maxPool2dBackward", "conv2dDevBias"} <= set(called)


@pytest.mark.parametrize("name,tol", [("tiny_cnn", 0.05), ("vgg_mini", 0.1)])
def test_pretrained_bundle_eval_on_oracle(tmp_path, name, tol):
    """The real-PyTorch pretrained bundles the reference's browser tests load
    (runtime/tests/browser.spec.ts:1088-1230): decoded by the reference's own
    torch.load, run in eval mode, the predictions equal the bundle's and the
    logits stay within the browser tests' bounds (0.05 / 0.1); on the oracle
    they are within 1e-4 of real PyTorch's."""
    out = tmp_path / "p.json"
    r = subprocess.run([sys.executable, os.path.join(HERE, "dropin_pretrained.py"), "oracle", name, str(out)],
                       capture_output=True, text=True, timeout=300, env=ENV)
    assert r.returncode == 0, r.stderr[-3000:]
    got = json.load(open(out))
    want = json.load(open(os.path.join(HERE, "golden", "pretrained", f"{name}.json")))["predictions"]
    assert got["preds"] == want["preds"]
    err = float(np.max(np.abs(np.asarray(got["logits"]) - np.asarray(want["logits"]))))
    assert err < tol and err <= 1e-4 * float(np.max(np.abs(want["logits"]))), err
