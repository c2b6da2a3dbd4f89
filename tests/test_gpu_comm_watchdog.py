"""The communicator watchdog (tp_comm_sync) and the host-side departure check,
tested without any collective or kernel left waiting for a lost rank: a rank
leaves only between steps and the other learns of it on the host (store mark)
before its next collective; the watchdog's own time limit is exercised with a
bounded device wait keeping the stream busy."""
import json
import os
import socket
import subprocess
import sys

import pytest

from tpcuda._lib import TpError, check

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
TP_ERR_TIMEOUT = -5


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def test_watchdog_times_out_while_the_stream_is_busy(cuda_rt):
    """One GPU, no communicator: tp_comm_sync(50 ms) gives up on a stream that a
    400 ms bounded wait keeps busy, and reports TP_ERR_TIMEOUT; the probe's own
    expired wait is reported by the next synchronize."""
    rt = cuda_rt
    rt.synchronize()
    check(rt.lib.tp_wait_probe(400_000_000))
    with pytest.raises(TpError) as e:
        check(rt.lib.tp_comm_sync(50))
    assert e.value.status == TP_ERR_TIMEOUT and "50 ms" in str(e.value)
    with pytest.raises(TpError):
        rt.synchronize()
    rt.synchronize()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_rank_leaving_between_steps_is_seen_and_watchdog_aborts(tmp_path):
    out = tmp_path / "w.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TPCUDA_STORE_DIR=str(tmp_path / "store"))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "comm_watchdog_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["first_sum"] == 3.0  # 1 + 2 over the two ranks
    assert res["departure"] and "[1]" in res["departure"]
    assert res["sync_status"] == TP_ERR_TIMEOUT and "aborted" in res["sync_msg"]
    assert res["world_after"] == 1
    assert res["probe_status"] == TP_ERR_TIMEOUT
