"""One rank of the data-parallel VGG-11-BN check, launched by
tests/test_gpu_dp.py through torch.distributed.run (one process per GPU; the
ranks meet through tpcuda.store, not torch.distributed).

Per rank, on its shard of a seeded global batch:
  1. a single-GPU model (no communicator) takes one eager step: its gradient
     buffer then holds this rank's local gradients;
  2. a data-parallel model (same init, NCCL communicator) takes one eager
     step: its gradient buffer then holds the bucketed all-reduce sum and its
     parameters the SGD update with the 1/world average folded in;
  3. the data-parallel model is captured into a CUDA graph (all-reduces
     included) and replayed a few steps.
Rank 0 writes the comparisons to the JSON file named by argv[1].
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "torch-pyodide_b200"))

import numpy as np  # noqa: E402

from tpcuda import CudaRuntime  # noqa: E402
from tpcuda.dp import comm_from_store, env_ranks  # noqa: E402
from tpcuda.store import FileStore  # noqa: E402
from tpcuda.vgg import VGG11BN  # noqa: E402

PER_RANK = 8
REPLAYS = 3


def main(out_path: str) -> None:
    rank, world, local = env_ranks()
    store = FileStore(rank, world, timeout_s=120)
    rt = CudaRuntime(local)
    comm = comm_from_store(rt.lib, store)

    def gather(vec: np.ndarray, world: int) -> list[np.ndarray]:
        return store.all_gather_array(vec)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((PER_RANK * world, 3, 32, 32)).astype(np.float32)[rank * PER_RANK:(rank + 1) * PER_RANK]
    y = rng.integers(0, 10, PER_RANK * world).astype(np.float32)[rank * PER_RANK:(rank + 1) * PER_RANK]

    loc = VGG11BN(rt, PER_RANK, seed=0)
    loc._h2d(loc.x, x)
    loc._h2d(loc.y, y)
    p0 = loc.read(loc.params, loc.flat_len)
    loc.step_eager()
    rt.synchronize()
    g_local = loc.read(loc.grads, loc.flat_len)
    loc.close()

    dp = VGG11BN(rt, PER_RANK, seed=0, world=world, comm=comm, bucket_bytes=4 << 20)
    dp._h2d(dp.x, x)
    dp._h2d(dp.y, y)
    dp.step_eager()
    comm.sync(60000)
    g_sum = dp.read(dp.grads, dp.flat_len)
    p1 = dp.read(dp.params, dp.flat_len)

    locals_ = gather(g_local, world)
    expect = locals_[0].copy()
    for g in locals_[1:]:
        expect = expect + g
    # SGD, first step (momentum buffer from zero): p - lr * (g / world + wd * p)
    p_expect = (p0.astype(np.float64) - dp.lr * (expect.astype(np.float64) / world + dp.wd * p0.astype(np.float64)))
    sums = gather(g_sum, world)
    params1 = gather(p1, world)

    dp.capture()
    for _ in range(REPLAYS):
        dp.step()
    comm.sync(60000)
    loss = dp.read_loss()
    params2 = gather(dp.read(dp.params, dp.flat_len), world)
    dp.close()
    comm.close()
    store.close()
    if rank == 0:
        scale = float(np.max(np.abs(expect)))
        res = {
            "world": world,
            "buckets": len(dp.buckets),
            "grad_sum_maxdiff": float(np.max(np.abs(g_sum - expect))),
            "grad_scale": scale,
            "grad_sum_rank_maxdiff": max(float(np.max(np.abs(s - sums[0]))) for s in sums),
            "update_maxdiff": float(np.max(np.abs(p1.astype(np.float64) - p_expect))),
            "param_scale": float(np.max(np.abs(p0))),
            "params_rank_maxdiff_step1": max(float(np.max(np.abs(p - params1[0]))) for p in params1),
            "params_rank_maxdiff_graph": max(float(np.max(np.abs(p - params2[0]))) for p in params2),
            "loss_after_graph_steps": loss,
        }
        with open(out_path, "w") as f:
            json.dump(res, f)


if __name__ == "__main__":
    main(sys.argv[1])
