"""The unmodified reference package, patched (tpcuda.patches), live on the CUDA
runtime, against the same scripts on the CPU oracle runtime.

* Training: the Tiny CNN config (Adam), a small CNN with every rebound op (SGD
  momentum, AdamW) and VGG-11-BN at batch 8 (SGD momentum 0.9, weight decay
  5e-4) train 3 steps through the reference's nn / autograd / optim with the
  CUDA runtime underneath; losses, first-step gradients and final parameters
  match the oracle run to 1e-4 of their scale (parameters whose gradient is
  mathematically zero -- conv biases feeding a BatchNorm -- excluded, as in
  the CPU cross-check against PyTorch), and the device memory the runtime holds
  is the same after every step (no leak of intermediates, D7).
* Pretrained real-PyTorch bundles (tiny_cnn, vgg_mini): eval predictions equal
  the bundle's, logits within the browser tests' bounds and within 1e-4 of the
  oracle's.

Runs only where the reference package travels with the repository
(baseline/_ref); each script runs in its own process.  These whole-program
runs (minutes of CPU oracle work) are named to be collected after the kernel
tests, so a run that stops at its first failure has checked every kernel.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from dropin_train import reference_path  # noqa: E402
from test_dropin_patches import compare, run_train  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(reference_path() is None, reason="reference package not installed (baseline/_ref)")]


@pytest.mark.parametrize("model,opt", [("tiny", "adam"), ("cnn", "sgd"), ("cnn", "adamw"), ("vgg", "sgd")])
def test_reference_package_trains_on_cuda_like_oracle(tmp_path, model, opt):
    cu = run_train("cuda", model, 3, tmp_path / "c.npz", opt)
    orc = run_train("oracle", model, 3, tmp_path / "o.npz", opt)
    compare(cu, orc)
    live = cu["live"]
    assert len(live) == 3 and live[0] == live[1] == live[2] > 0, live


def _pretrained(backend, name, out):
    r = subprocess.run([sys.executable, os.path.join(HERE, "dropin_pretrained.py"), backend, name, str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.load(open(out))


@pytest.mark.parametrize("name,tol", [("tiny_cnn", 0.05), ("vgg_mini", 0.1)])
def test_pretrained_bundle_eval_on_cuda(tmp_path, name, tol):
    cu = _pretrained("cuda", name, tmp_path / "c.json")
    orc = _pretrained("oracle", name, tmp_path / "o.json")
    want = json.load(open(os.path.join(HERE, "golden", "pretrained", f"{name}.json")))["predictions"]
    assert cu["preds"] == want["preds"] == orc["preds"]
    a, b, w = (np.asarray(v["logits"], np.float64) for v in (cu, orc, want))
    assert float(np.max(np.abs(a - w))) < tol
    assert float(np.max(np.abs(a - b))) <= 1e-4 * float(np.max(np.abs(b)))
    assert cu["keys"] == orc["keys"]


def test_trained_vgg_state_dict_checkpoint_roundtrip(tmp_path):
    """A VGG-11-BN trained 2 steps on the CUDA runtime, saved with the reference's
    torch.save (tensor bytes through tp_to_bytes) and loaded back with its
    torch.load (tp_from_bytes): every entry bit-exact, running statistics and
    num_batches_tracked included; real PyTorch loads the same file to the same
    values."""
    ckpt = tmp_path / "vgg.pt"
    env = dict(os.environ, DROPIN_CKPT=str(ckpt))
    res = run_train("cuda", "vgg", 2, tmp_path / "c.npz", "sgd", env=env)
    assert bool(res["ckpt_roundtrip_exact"])
    code = ("import json, torch; sd = torch.load(%r, weights_only=False); "
            "print(json.dumps({k: v.double().flatten().tolist() for k, v in sd.items()}))" % str(ckpt))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    real = json.loads(r.stdout.strip().splitlines()[-1])
    states = {k[len("state:"):]: res[k] for k in res.files if k.startswith("state:")}
    assert set(real) == set(states) and len(real) > 40
    for k, v in real.items():
        assert np.array_equal(np.asarray(v), states[k].ravel()), k
