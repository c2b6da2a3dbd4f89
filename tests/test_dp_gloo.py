"""Data-parallel host logic on CPU (no GPU): the flat parameter layout, the
gradient bucket plan, and a two-rank gloo run of the bucketed gradient
all-reduce in the order the VGG step issues it.

The device path issues exactly this sequence through NCCL (tpcuda.vgg
VGG11BN._reduce after each block's weight gradient, VGG11BN._update waits,
then the fused SGD applies 1/world); here each rank's local gradients come
from the oracle on its shard of a global batch, the buckets are all-reduced
with gloo, and rank 0 checks the result against the sum of both shards'
gradients computed in one process.
"""
import datetime
import os
import socket

import numpy as np
import pytest

from tpcuda.vgg import NUM_CLASSES, init_params, plan_blocks, plan_buckets, plan_params

GLOBAL_BATCH = 4
BUCKET_BYTES = 1 << 20  # small, so the plan has many buckets


def _layout():
    blocks = plan_blocks()
    specs, offsets, flat_len = plan_params(blocks, 512)
    return blocks, specs, offsets, flat_len


def test_plan_blocks_vgg11():
    blocks = plan_blocks()
    assert [(b["cin"], b["cout"], b["H"], b["pool"]) for b in blocks] == [
        (3, 64, 32, True), (64, 128, 16, True), (128, 256, 8, False), (256, 256, 8, True),
        (256, 512, 4, False), (512, 512, 4, True), (512, 512, 2, False), (512, 512, 2, True)]


def test_param_layout_aligned_and_disjoint():
    _, specs, offsets, flat_len = _layout()
    spans = sorted(offsets.values())
    for (o, n), (o2, _) in zip(spans, spans[1:]):
        assert o % 64 == 0 and o + n <= o2
    assert spans[-1][0] + spans[-1][1] <= flat_len and flat_len % 64 == 0
    assert sum(n for _, n in spans) == 9231114  # VGG-11-BN (CIFAR head) parameter count
    assert offsets["fc.w"][1] == NUM_CLASSES * 512


@pytest.mark.parametrize("bucket_bytes", [1, 1 << 20, 8 << 20, 1 << 40])
def test_buckets_cover_flat_buffer_once_in_backward_order(bucket_bytes):
    blocks, specs, offsets, flat_len = _layout()
    buckets = plan_buckets(offsets, len(blocks), flat_len, bucket_bytes)
    pos = 0
    for start, count, _ in buckets:
        assert start == pos and count > 0
        pos += count
    assert pos == flat_len
    order = ["fc"] + [f"blk{li}" for li in reversed(range(len(blocks)))]
    keys = [k for _, _, k in buckets]
    assert keys == sorted(keys, key=order.index)
    assert keys[-1] == "blk0"
    # a bucket closes only after every tensor in it has its final gradient
    done_after = {"fc.w": "fc", "fc.b": "fc"}
    for li in range(len(blocks)):
        for t in ("bn", "conv"):
            for s in ("g", "b", "w"):
                name = f"{t}{li}.{s}"
                if name in offsets:
                    done_after[name] = f"blk{li}"
    for name, (o, n) in offsets.items():
        owner = [k for s0, c, k in buckets if s0 <= o < s0 + c]
        assert len(owner) == 1 and o + n <= [s0 + c for s0, c, k in buckets if k == owner[0]][0]
        assert order.index(owner[0]) >= order.index(done_after[name]), name
    if bucket_bytes == 1:
        assert len(buckets) == 1 + len(blocks)
    if bucket_bytes == 1 << 40:
        assert buckets == [(0, flat_len, "blk0")]


def _shard_grads(orc, blocks, specs, offsets, flat_len, rank, world):
    from vgg_oracle import oracle_grads

    class _Model:
        pass

    model = _Model()
    model.blocks = blocks
    host = init_params(specs, offsets, flat_len, 0)
    params = {n: (host[offsets[n][0]:offsets[n][0] + offsets[n][1]], s) for n, s, _ in specs}
    rng = np.random.default_rng(7)
    x = rng.standard_normal((GLOBAL_BATCH, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, GLOBAL_BATCH).astype(np.float32)
    b = GLOBAL_BATCH // world
    stats = [(np.zeros(bl["cout"], np.float32), np.ones(bl["cout"], np.float32)) for bl in blocks]
    _, grads = oracle_grads(orc, model, params, x[rank * b:(rank + 1) * b], y[rank * b:(rank + 1) * b], stats)
    flat = np.zeros(flat_len, np.float32)
    for n, (o, k) in offsets.items():
        flat[o:o + k] = grads[n]
    return flat


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from oracle_runtime import OracleRuntime

        orc = OracleRuntime()
        blocks, specs, offsets, flat_len = _layout()
        buckets = plan_buckets(offsets, len(blocks), flat_len, BUCKET_BYTES)
        bucket_after = {k: (s, c) for s, c, k in buckets}
        flat = _shard_grads(orc, blocks, specs, offsets, flat_len, rank, world)
        local = flat.copy()
        grads = torch.from_numpy(flat)
        # backward order: fc, then blocks last to first; each closing bucket is
        # reduced asynchronously, all are waited for before the update
        works = []
        for key in ["fc"] + [f"blk{li}" for li in reversed(range(len(blocks)))]:
            if key in bucket_after:
                s, c = bucket_after[key]
                works.append(dist.all_reduce(grads[s:s + c], async_op=True))
        for w in works:
            w.wait()
        summed = grads.numpy()
        if rank == 0:
            other = _shard_grads(orc, blocks, specs, offsets, flat_len, 1, world)
            expect = local + other
            q.put(("ok", float(np.max(np.abs(summed - expect))), len(buckets),
                   float(np.max(np.abs(local))), float(np.max(np.abs(other)))))
        dist.barrier()
    except Exception as e:  # reported to the parent, which fails the test
        q.put(("error", f"rank {rank}: {e!r}"))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_bucketed_allreduce_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    msg = q.get(timeout=5)
    assert msg[0] == "ok", msg
    _, diff, nbuckets, m0, m1 = msg
    assert nbuckets > 3
    assert m0 > 0 and m1 > 0
    assert diff == 0.0  # a + b in fp32 is the same on either rank and in numpy
