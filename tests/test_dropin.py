"""Drop-in boundary: the shim modules, and the runtime surface the reference
package calls (python/torch/_runtime.py:15-39)."""
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = "/root/reference"

# runtime.ts methods on the hot path (matmul/linear, conv2d fwd/bwd, pooling,
# reductions, softmax, norms, element-wise chains, optimizer steps, creation,
# shape, readback).
HOT = """tensorFromData zeros ones full fullLike zerosLike onesLike emptyLike empty fill setSeed rand randn
add sub mul div pow mulScalar relu rsqrt neg gt expand reshape flatten squeeze unsqueeze transpose2d transpose
permute matmul sum mean sumDim meanDim max argmax softmax logSoftmax softmaxBackward logSoftmaxBackward
crossEntropy crossEntropyBackward conv2d conv2dInputBackward conv2dWeightBackward conv2dBiasBackward maxPool2d
batchNorm layerNorm adamStep adamWStep sgdStep beginFrame endFrame toList destroy init isAvailable
deviceCount""".split()


def test_shim_installs_runtime():
    from tpcuda import shim

    class Dummy:
        pass

    d = Dummy()
    shim.install(d)
    try:
        from js import globalThis  # noqa: F401
        from pyodide.ffi import can_run_sync, run_sync
        assert getattr(globalThis, "__torch_pyodide_runtime__") is d
        assert can_run_sync() and run_sync(5) == 5
    finally:
        shim.uninstall()


def test_cuda_runtime_implements_hot_surface():
    from tpcuda.runtime import CudaRuntime
    missing = [m for m in HOT if not callable(getattr(CudaRuntime, m, None))]
    assert not missing, missing


def test_oracle_runtime_implements_hot_surface():
    from oracle_runtime import OracleRuntime
    missing = [m for m in HOT if not callable(getattr(OracleRuntime, m, None))]
    assert not missing, missing


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="reference checkout not mounted")
def test_hot_surface_is_what_the_reference_calls():
    """Every hot method is one the reference Python actually calls (the regex
    of runtime/scripts/validate-runtime-api.mjs:14-45)."""
    called = set()
    for dirpath, _, files in os.walk(os.path.join(REFERENCE, "python", "torch")):
        for f in files:
            if f.endswith(".py"):
                text = open(os.path.join(dirpath, f)).read()
                called |= set(re.findall(r"runtime(?:\(\))?\.(\w+)\s*\(", text))
                # unary ops dispatched by name: getattr(runtime, fn_name) (tensor_ops.py:1226-1230)
                called |= set(re.findall(r"_make_unary_from_tensor\(\"(\w+)\"\)", text))
    not_called = [m for m in HOT if m not in called and m not in ("init", "transpose2d")]
    assert not not_called, not_called


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="reference checkout not mounted")
def test_reference_package_runs_unedited_on_oracle_via_shim():
    code = f"""
import sys
sys.path.insert(0, {os.path.join(ROOT, 'torch-pyodide_b200')!r}); sys.path.insert(0, {os.path.join(ROOT, 'oracle')!r})
from tpcuda import shim
from oracle_runtime import OracleRuntime
shim.install(OracleRuntime())
sys.path.insert(0, {os.path.join(REFERENCE, 'python')!r})
import torch
a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], requires_grad=True)
loss = a.mul(a).sum(); loss.backward()
print(loss.item(), a.grad.tolist())
"""
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split()[0] == "30.0"
