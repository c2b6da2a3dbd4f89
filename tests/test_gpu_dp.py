"""Data-parallel VGG-11-BN on 2+ GPUs: the bucketed NCCL all-reduce sums the
ranks' local gradients exactly, every rank applies the same averaged SGD
update, and the graph-captured step (all-reduces inside the graph) keeps the
replicas identical.  Runs tests/dp_worker.py under torch.distributed.run;
skipped on a machine with fewer than two GPUs."""
import json
import math
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_dp_two_ranks(tmp_path):
    out = tmp_path / "dp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(HERE, "dp_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["buckets"] >= 3
    # the sum of two fp32 values is the same whichever rank adds it
    assert res["grad_sum_maxdiff"] == 0.0 and res["grad_scale"] > 0
    assert res["grad_sum_rank_maxdiff"] == 0.0
    assert res["update_maxdiff"] <= 1e-6 * max(1.0, res["param_scale"])
    assert res["params_rank_maxdiff_step1"] == 0.0
    assert res["params_rank_maxdiff_graph"] == 0.0
    assert math.isfinite(res["loss_after_graph_steps"])
