"""Eval of a real-PyTorch pretrained bundle through the unmodified reference
package (with tpcuda.patches) on the oracle or the CUDA runtime: the
state_dict is decoded with the reference's own torch.load (PyTorch's zipfile
format), loaded into the bundle's architecture, and run in eval mode on the
bundle's sample input.  The two architectures are those of the reference's
pretrained examples (runtime/playground/public/examples/
real_model_pretrained_tiny_cnn.py and real_model_pretrained_vgg.py), restated.

  python dropin_pretrained.py <oracle|cuda> <tiny_cnn|vgg_mini> <out.json>
"""
import base64
import io
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main():
    backend, name, out = sys.argv[1:4]
    sys.path[:0] = [os.path.join(ROOT, "torch-pyodide_b200"), os.path.join(ROOT, "oracle"), HERE]
    from dropin_train import reference_path
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
    patches.apply()

    class TinyCNN(nn.Module):
        def __init__(self):
            super().__init__()
            self.conv1 = nn.Conv2d(3, 8, kernel_size=3, padding=1)
            self.conv2 = nn.Conv2d(8, 16, kernel_size=3, padding=1)
            self.fc1 = nn.Linear(16 * 4 * 4, 32)
            self.fc2 = nn.Linear(32, 5)

        def forward(self, x):
            x = F.max_pool2d(F.relu(self.conv1(x)), 2)
            x = F.max_pool2d(F.relu(self.conv2(x)), 2)
            return self.fc2(F.relu(self.fc1(x.flatten(1))))

    class MiniVGG(nn.Module):
        def __init__(self):
            super().__init__()
            self.conv1, self.bn1 = nn.Conv2d(3, 16, 3, padding=1), nn.BatchNorm2d(16)
            self.conv2, self.bn2 = nn.Conv2d(16, 32, 3, padding=1), nn.BatchNorm2d(32)
            self.conv3, self.bn3 = nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64)
            self.fc1, self.fc2 = nn.Linear(64 * 2 * 2, 64), nn.Linear(64, 5)
            self.dropout = nn.Dropout(0.5)

        def forward(self, x):
            x = F.max_pool2d(F.relu(self.bn1(self.conv1(x))), 2)
            x = F.max_pool2d(F.relu(self.bn2(self.conv2(x))), 2)
            x = F.max_pool2d(F.relu(self.bn3(self.conv3(x))), 2)
            return self.fc2(self.dropout(F.relu(self.fc1(x.flatten(1)))))

    bundle = json.load(open(os.path.join(HERE, "golden", "pretrained", f"{name}.json")))
    sd = torch.load(io.BytesIO(base64.b64decode(bundle["state_dict_b64"])), weights_only=False)
    model = TinyCNN() if name == "tiny_cnn" else MiniVGG()
    model.load_state_dict(sd)
    model.eval()
    x = torch.tensor(bundle["sample_x"])
    with torch.no_grad():
        logits = model(x)
        probs = logits.softmax(dim=-1)
        preds = probs.argmax(dim=-1)
    json.dump({"logits": logits.tolist(), "probs": probs.tolist(), "preds": [int(p) for p in preds.tolist()],
               "keys": sorted(sd.keys())}, open(out, "w"))


if __name__ == "__main__":
    main()
