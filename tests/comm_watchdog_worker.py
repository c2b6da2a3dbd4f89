"""One rank of the communicator-watchdog check (tests/test_gpu_comm_watchdog.py),
launched under torch.distributed.run with NCCL_NVLS_ENABLE=0.

Both ranks build the NCCL communicator through the file store and complete one
all-reduce step.  Then rank 1 leaves between steps (no collective in flight:
it leaves a store mark, destroys its communicator and exits).  Rank 0 learns of it on the host before its
next step, so it issues no collective that would wait for rank 1; it then keeps
its library stream busy with a bounded device wait (tp_wait_probe, 400 ms) and
calls the watchdog tp_comm_sync with a 50 ms limit, which must give up with
TP_ERR_TIMEOUT and abort the communicator (tp_comm_info then reports one
rank).  Rank 0 writes what it saw to argv[1].
"""
import ctypes
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "torch-pyodide_b200"))

import numpy as np  # noqa: E402

from tpcuda import CudaRuntime  # noqa: E402
from tpcuda._lib import TpError, check  # noqa: E402
from tpcuda.dp import comm_from_store, env_ranks  # noqa: E402
from tpcuda.store import FileStore  # noqa: E402


def main(out_path):
    rank, world, local = env_ranks()
    store = FileStore(rank, world, timeout_s=120)
    rt = CudaRuntime(local)
    comm = comm_from_store(rt.lib, store)
    x = rt.tensorFromData(np.full(1 << 20, rank + 1, np.float32), [1 << 20], "float32")
    comm.allreduce_async(rt.devicePtr(x["id"]), 1 << 20)
    comm.wait()
    comm.sync(30000)
    first = float(rt.toNumpy(x["id"])[0])
    store.barrier()
    if rank == 1:
        # nothing in flight: leave the mark first (destroying the communicator
        # can wait for the peer's own teardown), then release it and exit
        store.leave()
        comm.close()
        return
    seen = None
    for _ in range(2000):  # the next step's check, before any collective
        try:
            comm.check_peers(store)
        except RuntimeError as e:
            seen = str(e)
            break
        import time
        time.sleep(0.005)
    check(rt.lib.tp_wait_probe(400_000_000))
    status, msg = 0, ""
    try:
        comm.sync(50)
    except TpError as e:
        status, msg = e.status, str(e)
    world_after = comm.world_now()
    try:
        rt.synchronize()  # the probe's own expired wait is reported here, once
        probe_status = 0
    except TpError as e:
        probe_status = e.status
    json.dump({"first_sum": first, "departure": seen, "sync_status": status, "sync_msg": msg,
               "world_after": world_after, "probe_status": probe_status}, open(out_path, "w"))


if __name__ == "__main__":
    main(sys.argv[1])
