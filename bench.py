#!/usr/bin/env python3
"""Benchmark of the B200 backend for the torch-pyodide hot path.

Default workload (every --gpus N): the VGG-11-BN data-parallel training step,
global batch 1024 split over the ranks (1024/N images per rank), SGD momentum
0.9, weight decay 5e-4, lr 0.05; input [B,3,32,32] ~N(0,1), labels uniform in
[0,10).  One step = forward, backward, the bucketed NCCL gradient all-reduce
overlapped with backward, and the fused SGD update, replayed as one CUDA
graph per rank.  value = 1024 images / the slowest rank's step time.

At N = 1 the same JSON line also carries, under "adamw", the other half of the
headline metric: the fused AdamW optimizer step over 64 parameter tensors
cycling [4096,4096], [4096], [1024,4096], [4096,1024] (402,718,720 fp32
elements; params ~N(0,0.02), grads ~N(0,1e-3), moments zero-initialised and
warmed for 3 steps), one multi-tensor launch per step, 28 B of HBM traffic per
element (read param, grad, exp_avg, exp_avg_sq; write param, exp_avg,
exp_avg_sq).  Its working set (11.3 GB per step) is ~90x the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload vgg|adamw|ops|conv|tiny]

--impl reference times the reference algorithm on the host cores (the oracle:
a C/OpenMP restatement of the reference's WGSL shaders, which cannot run here
without a WebGPU device) for the same workload and metric; under torchrun only
rank 0 runs it.  Ranks meet through tpcuda.store (a file rendezvous), not
torch.distributed.  Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "torch-pyodide_b200"))

SHAPES = [[4096, 4096], [4096], [1024, 4096], [4096, 1024]]
NTENSORS = 64
BYTES_PER_ELEM = 28
LR, B1, B2, EPS, WD = 1e-3, 0.9, 0.999, 1e-8, 0.01


def numel(s):
    r = 1
    for v in s:
        r *= v
    return r


def adam_scalars(step):
    bc1 = 1.0 - B1 ** step
    bc2 = 1.0 - B2 ** step
    return LR / bc1, 1.0 / math.sqrt(bc2)  # optim/__init__.py:385-388


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) taken while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}: launch with torchrun --nproc-per-node {gpus}")
    return rank, world, local


def make_store(rank, world):
    """The ranks' rendezvous (tpcuda.store): NCCL unique id, barriers, max over ranks."""
    from tpcuda.store import FileStore
    return FileStore(rank, world, timeout_s=300)


# ---------------------------------------------------------------------------
# CPU arms: the oracle (a C/OpenMP restatement of adamw_step.wgsl)

def cpu_adamw(sample_tensors: int, steps: int, warmup: int = 1) -> dict:
    """Time the oracle's AdamW on the first `sample_tensors` tensors of the
    workload (64 = the whole workload) with the host threads OMP_NUM_THREADS
    allows; returns GB/s of algorithmic traffic (28 B per element)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle_runtime as O
    L = O.lib()
    rng = np.random.default_rng(0)
    ts = []
    for i in range(sample_tensors):
        n = numel(SHAPES[i % 4])
        p = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))
        g = (rng.standard_normal(n, dtype=np.float32) * np.float32(1e-3))
        ts.append((p, g, np.zeros(n, np.float32), np.zeros(n, np.float32)))
    elems = sum(t[0].size for t in ts)

    def step(k):
        ss, isb = adam_scalars(k)
        for p, g, m, v in ts:
            L.or_adamw_step(O.fp(p), O.fp(g), O.fp(m), O.fp(v), p.size, LR, B1, B2, EPS, WD, ss, isb)

    for k in range(max(1, warmup)):
        step(k + 1)
    times = []
    for k in range(steps):
        t0 = time.perf_counter()
        step(k + 1 + max(1, warmup))
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"gbs": BYTES_PER_ELEM * elems / t / 1e9, "elems": elems, "sec": t, "times": times}


VGG_CPU_BATCH = 16  # images per oracle step: the bounded CPU sample of the 1024-image step


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm of the same workload on the
    host cores (the reference's WGSL shaders cannot run here: there is no
    WebGPU device; the oracle restates their arithmetic in C/OpenMP), same
    metric, unit and config.  Rank 0 alone runs it."""
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    steps, warmup = max(1, args.steps), max(1, args.warmup)
    if args.workload == "tiny":
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle_runtime import OracleRuntime
        orc = OracleRuntime()
        calls = json.load(open(TINY_TRACE))["calls"]
        for _ in range(max(1, warmup // 10)):
            replay_trace(orc, calls)
        t = []
        for _ in range(max(1, steps // 10)):
            t += replay_trace(orc, calls)[0]
        ms = statistics.median(t) * 1e3
        line = {"impl": "reference", "metric": "Tiny CNN train step (replayed reference runtime-call stream)",
                "value": round(ms, 4), "unit": "ms/step", "n_gpus": args.gpus, "steps": len(t),
                "warmup": 10 * max(1, warmup // 10), "ms_per_step": round(ms, 4), "higher_is_better": False,
                "scaling": "replicas only", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "Tiny CNN, batch 64, Adam lr 1e-3, 10 recorded steps per replay"},
                "cpu_baseline": {"value": round(ms, 4), "unit": "ms/step", "cores": cores, "kind": "port",
                                 "sample": "the recorded 10-step stream on the oracle runtime"},
                "e2e": {"value": round(ms, 4), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    elif args.workload == "adamw":
        r = cpu_adamw(NTENSORS, steps, warmup)
        elems = r["elems"]
        line = {
            "impl": "reference", "metric": "fused AdamW HBM GB/s", "value": round(r["gbs"], 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "ms_per_step": round(r["sec"] * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": ADAMW_WORKLOAD, "same_config": True, "elements": elems},
            "cpu_baseline": {"value": round(r["gbs"], 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"all 64 tensors ({elems} elements), median of {len(r['times'])} steps"},
            "e2e": {"value": round(r["gbs"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    else:
        r = cpu_vgg(VGG_CPU_BATCH, steps, warmup)
        line = {
            "impl": "reference", "metric": "VGG-11-BN train imgs/s", "value": round(r["imgs_per_s"], 4),
            "unit": "imgs/s", "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
            "ms_per_step": round(r["sec"] * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": VGG_WORKLOAD, "global_batch": VGG_GLOBAL_BATCH,
                       "sample": f"{VGG_CPU_BATCH} images per step (model resident, SGD each step)"},
            "cpu_baseline": {"value": round(r["imgs_per_s"], 4), "unit": "imgs/s", "cores": cores, "kind": "port",
                             "sample": f"oracle VGG-11-BN step at batch {VGG_CPU_BATCH}, median of {steps} steps"},
            "e2e": {"value": round(r["imgs_per_s"], 4), "unit": "imgs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# The fused AdamW step (device-resident and end to end)

ADAMW_WORKLOAD = "adamw 64 tensors cycling [4096,4096],[4096],[1024,4096],[4096,1024]"


def measure_adamw(args, rt, rank, world, store, ntensors):
    """Build the 64-tensor AdamW workload with the library's own creation
    kernels, warm the moments for 3 steps, then time --steps fused launches
    (device-resident) and end-to-end steps (grads copied from pinned host
    memory through the C ABI, one value read back).  Returns a dict."""
    import ctypes

    import numpy as np
    import torch
    from tpcuda._lib import check
    lib = rt.lib
    stream = torch.cuda.ExternalStream(rt.stream(), device=torch.device("cuda", torch.cuda.current_device()))
    rt.setSeed(1000 + rank)
    P, G, M, V = [], [], [], []
    for i in range(ntensors):
        s = SHAPES[i % 4]
        P.append(rt.normal(s, "float32", 0.0, 0.02))
        G.append(rt.normal(s, "float32", 0.0, 1e-3))
        M.append(rt.zeros(s, "float32"))
        V.append(rt.zeros(s, "float32"))
    elems = sum(numel(h["shape"]) for h in P)
    ptr = lambda hs: (ctypes.c_void_p * len(hs))(*[rt.devicePtr(h["id"]) for h in hs])  # noqa: E731
    numels = (ctypes.c_int64 * ntensors)(*[numel(h["shape"]) for h in P])
    group = ctypes.c_int64(0)
    check(lib.tpk_group_create(ntensors, ptr(P), ptr(G), ptr(M), ptr(V), numels, ctypes.byref(group)))
    step_no = [0]

    def step():
        step_no[0] += 1
        ss, isb = adam_scalars(step_no[0])
        check(lib.tpk_adam_group(group.value, 0, LR, B1, B2, EPS, WD, ss, isb))

    # 3 warm steps of the moments with regenerated grads (seed + step)
    for k in range(3):
        for h in G:
            rt.destroy(h["id"])
        rt.setSeed(2000 + 97 * rank + k)
        G = [rt.normal(SHAPES[i % 4], "float32", 0.0, 1e-3) for i in range(ntensors)]
        check(lib.tpk_group_destroy(group.value))
        check(lib.tpk_group_create(ntensors, ptr(P), ptr(G), ptr(M), ptr(V), numels, ctypes.byref(group)))
        step()
    for _ in range(args.warmup):
        step()
    rt.synchronize()

    def barrier():
        rt.synchronize()
        store.barrier()

    clocks = ClockSampler(torch.cuda.current_device())
    barrier()
    clocks.start()
    launches0 = rt.kernelLaunches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    launches = rt.kernelLaunches() - launches0
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_step = store.max(ms) / args.steps
    total_bytes = BYTES_PER_ELEM * elems * world
    value = total_bytes / (ms_step * 1e-3) / 1e9
    kernel_gbs = BYTES_PER_ELEM * elems / (ms / args.steps * 1e-3) / 1e9

    # ---- end to end through the handle-level C ABI, grads from pinned host ----
    host_g = [torch.empty(numel(SHAPES[i % 4]), dtype=torch.float32, pin_memory=True) for i in range(ntensors)]
    for hg in host_g:
        hg.normal_(0.0, 1e-3)
    ids = lambda hs: [h["id"] for h in hs]  # noqa: E731
    gptr = [rt.devicePtr(h["id"]) for h in G]
    readback = np.zeros(1, np.float32)
    h2d = sum(hg.numel() * 4 for hg in host_g)
    e2e_steps = max(2, min(args.steps, 10))

    def e2e_step():
        for i, hg in enumerate(host_g):
            check(lib.tp_memcpy_h2d(ctypes.c_void_p(gptr[i]), ctypes.c_void_p(hg.data_ptr()), hg.numel() * 4))
        step_no[0] += 1
        ss, isb = adam_scalars(step_no[0])
        rt.adamWStepMulti(ids(P), ids(G), ids(M), ids(V), LR, B1, B2, EPS, WD, ss, isb)
        check(lib.tp_memcpy_d2h(readback.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(rt.devicePtr(P[0]["id"])),
                                4))

    e2e_step()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(stream)
    f1.synchronize()
    e2e_ms = store.max(f0.elapsed_time(f1)) / e2e_steps
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    check(lib.tpk_group_destroy(group.value))
    for h in P + G + M + V:
        rt.destroy(h["id"])
    del host_g
    rt.synchronize()
    peak, peak_kind = measured_peaks()
    rec = {
        "metric": "fused AdamW HBM GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ADAMW_WORKLOAD, "elements_per_rank": elems, "bytes_per_element": BYTES_PER_ELEM,
                   "l2": "working set 11.3 GB per step >> 126 MB L2, no flush",
                   "parallelism": f"replicas x{world}", "lr": LR, "betas": [B1, B2], "eps": EPS,
                   "weight_decay": WD},
        "gpu_launches": int(launches),
        "clocks": clk,
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(kernel_gbs / peak, 4), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "k_adam_multi<true>"},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "path": "tp_memcpy_h2d(pinned grads) + tp_adamw_step_multi(ids) + tp_memcpy_d2h"},
    }
    tf = os.path.join(ROOT, "profiles", "adamw_traffic.json")
    if os.path.exists(tf):
        rec["roofline"]["traffic"] = json.load(open(tf)).get("bytes_per_launch")
    return rec


def adamw_cpu_baseline():
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    r = cpu_adamw(8, 5)
    return {"value": round(r["gbs"], 3), "unit": "GB/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
            "kind": "port", "sample": f"oracle AdamW on 8 of 64 tensors ({r['elems']} elements), median of 5 steps"}


def run_ours(args, rank, world, local):
    """--workload adamw: the fused AdamW step alone (N replicas for --gpus N)."""
    import torch
    torch.cuda.set_device(local)
    from tpcuda import CudaRuntime
    rt = CudaRuntime(local)
    store = make_store(rank, world)
    line = measure_adamw(args, rt, rank, world, store, args.tensors)
    store.close()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = adamw_cpu_baseline()
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# VGG-11-BN data-parallel training: global batch 1024 split over the ranks

VGG_GLOBAL_BATCH = 1024
VGG_WORKLOAD = ("vgg11-bn train step, x[B,3,32,32]~N(0,1), y~U{0..9}, SGD mom 0.9 wd 5e-4 lr 0.05, "
                "global batch 1024")


def tf32x3_peak():
    """3xTF32 dense peak derived from the measured bf16 GEMM rate: TF32 runs at
    half the bf16 rate on Blackwell tensor cores and 3xTF32 issues three MMAs
    per product."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]) / 2 / 3, float(d["bf16_tflops"]), "measured"
    return 1590.0 / 2 / 3, 1590.0, "fallback"


def vgg_plan_cpu():
    """The VGG-11-BN block plan (tpcuda.vgg's) built without touching the GPU."""
    class Plan:
        blocks = []

    cfg = [64, "M", 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"]
    cin, H, i = 3, 32, 0
    while i < len(cfg):
        pool = i + 1 < len(cfg) and cfg[i + 1] == "M"
        Plan.blocks.append({"cin": cin, "cout": cfg[i], "H": H, "W": H, "pool": pool})
        cin = cfg[i]
        H = H // 2 if pool else H
        i += 2 if pool else 1
    return Plan


def cpu_vgg_trainer(batch: int, seed: int = 0):
    """The oracle composition of the VGG-11-BN training step (conv, BN train,
    ReLU, max-pool with indices, linear, cross-entropy, their backward rules,
    multi-tensor SGD momentum 0.9 wd 5e-4 lr 0.05), model resident in the
    oracle runtime; returns (trainer, x, y) for a seeded batch."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    from oracle_runtime import OracleRuntime
    from vgg_oracle import OracleTrainer

    Plan = vgg_plan_cpu()
    rng = np.random.default_rng(seed)
    params = {"fc.w": (rng.uniform(-0.04, 0.04, 5120).astype(np.float32), [10, 512]),
              "fc.b": (np.zeros(10, np.float32), [10])}
    stats = []
    for li, b in enumerate(Plan.blocks):
        bound = 1 / (b["cin"] * 9) ** 0.5
        params[f"conv{li}.w"] = (rng.uniform(-bound, bound, b["cout"] * b["cin"] * 9).astype(np.float32),
                                 [b["cout"], b["cin"], 3, 3])
        params[f"conv{li}.b"] = (np.zeros(b["cout"], np.float32), [b["cout"]])
        params[f"bn{li}.g"] = (np.ones(b["cout"], np.float32), [b["cout"]])
        params[f"bn{li}.b"] = (np.zeros(b["cout"], np.float32), [b["cout"]])
        stats.append((np.zeros(b["cout"], np.float32), np.ones(b["cout"], np.float32)))
    x = rng.standard_normal((batch, 3, 32, 32)).astype(np.float32)
    y = rng.integers(0, 10, batch).astype(np.float32)
    return OracleTrainer(OracleRuntime(), Plan, params, stats, 0.05, 0.9, 5e-4), x, y


def cpu_vgg(batch: int, steps: int, warmup: int = 1) -> dict:
    """Time the oracle's VGG-11-BN training step at `batch` images on the host
    cores (OpenMP threads = OMP_NUM_THREADS); median over `steps` timed steps."""
    tr, x, y = cpu_vgg_trainer(batch)
    for _ in range(warmup):
        tr.step(x, y)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        tr.step(x, y)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"imgs_per_s": batch / t, "sec": t, "batch": batch, "times": times}


def cpu_ops(reps: int = 3) -> dict:
    """The oracle (C/OpenMP restatement of the reference shaders, all host
    threads) on the reductions / norms and dense configs: per op the same rate
    the GPU line reports (GB/s of algorithmic traffic, or TFLOP/s), measured on
    the full input where the oracle takes seconds, else on a stated sample of
    the output (rows of a matmul, whole images of a convolution, output
    channels of a weight gradient) -- each sampled output value is computed as
    in the full op, so the rate carries over.  Keyed by the GPU line's op names."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    from oracle_runtime import OracleRuntime
    o = OracleRuntime()
    rng = np.random.default_rng(0)
    res = {}

    def T(a):
        a = np.ascontiguousarray(a, np.float32)
        return o.tensorFromData(a.ravel(), list(a.shape), "float32")["id"]

    def best(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            out = fn()
            ts.append(time.perf_counter() - t0)
            for h in (out if isinstance(out, list) else [out]):
                if isinstance(h, dict):
                    o.destroy(h["id"])
        return statistics.median(ts)

    def put(name, sec, work, kind, sample="full size"):
        rate = work / sec / (1e9 if kind == "hbm" else 1e12)
        res[name] = {"value": round(rate, 4), "unit": "GB/s" if kind == "hbm" else "TFLOP/s",
                     "ms": round(sec * 1e3, 3), "sample": sample}

    x = T(rng.standard_normal((16384, 4096), dtype=np.float32))
    g, b = T(np.ones(4096)), T(np.zeros(4096))
    nb = 16384 * 4096 * 4
    put("layer_norm fwd", best(lambda: o.layerNormForward(x, [4096], g, b, 1e-5)), 2 * nb, "hbm")
    y, m, r = o.layerNormForward(x, [4096], g, b, 1e-5)
    put("layer_norm bwd", best(lambda: o.layerNormBackward(x, x, [4096], g, m["id"], r["id"])), 3 * nb, "hbm")
    for h in (x, g, b, y["id"], m["id"], r["id"]):
        o.destroy(h)
    x = T(rng.standard_normal((32768, 8192), dtype=np.float32))
    nb = 32768 * 8192 * 4
    put("softmax", best(lambda: o.softmax(x, -1)), 2 * nb, "hbm")
    put("log_softmax", best(lambda: o.logSoftmax(x, -1)), 2 * nb, "hbm")
    # the backward as the reference computes it is O(C^2) per row: 64 of the rows
    xs = T(rng.standard_normal((64, 8192), dtype=np.float32))
    s = o.softmax(xs, -1)["id"]
    nbs = 64 * 8192 * 4
    put("softmax bwd", best(lambda: o.softmaxBackward(xs, s, 64, 8192)), 3 * nbs, "hbm", "64 of 32768 rows")
    put("log_softmax bwd", best(lambda: o.logSoftmaxBackward(xs, s, 64, 8192)), 3 * nbs, "hbm", "64 of 32768 rows")
    o.destroy(s)
    o.destroy(xs)
    o.destroy(x)
    x = T(rng.standard_normal((8192, 8192), dtype=np.float32))
    nb = 8192 * 8192 * 4
    put("sum all", best(lambda: o.sum(x)), nb, "hbm")
    for d in (0, -1):
        put(f"sum dim {d}", best(lambda: o.sumDim(x, d, False)), nb, "hbm")
        put(f"mean dim {d}", best(lambda: o.meanDim(x, d, False)), nb, "hbm")
        put(f"max dim {d}", best(lambda: o.maxDim(x, d, False)), nb, "hbm")
    o.destroy(x)
    shp = [256, 128, 56, 56]
    x = T(rng.standard_normal(shp, dtype=np.float32))
    g, b, rm, rv = T(np.ones(128)), T(np.zeros(128)), T(np.zeros(128)), T(np.ones(128))
    nb = 256 * 128 * 56 * 56 * 4
    put("batch_norm train fwd", best(lambda: o.batchNormTrain(x, g, b, rm, rv, 1e-5, 0.1)), 2 * nb, "hbm")
    _, mean, inv = o.batchNormTrain(x, g, b, rm, rv, 1e-5, 0.1)
    put("batch_norm bwd", best(lambda: o.batchNormBackward(x, x, g, mean["id"], inv["id"])), 3 * nb, "hbm")
    for h in (x, g, b, rm, rv):
        o.destroy(h)
    for n, rows in ((512, 512), (2048, 128), (8192, 16)):
        a, bb = rng.uniform(-1, 1, (rows, n)).astype(np.float32), rng.uniform(-1, 1, (n, n)).astype(np.float32)
        ta, tb = T(a), T(bb)
        put("matmul", best(lambda: o.matmul(ta, tb)), 2.0 * rows * n * n, "tensor",
            "full size" if rows == n else f"{rows} of {n} output rows")
        res[f"matmul {n}"] = res.pop("matmul")
        o.destroy(ta)
        o.destroy(tb)
    xl = T(rng.uniform(-1, 1, (16, 4096)).astype(np.float32))
    wt = o.transpose2d(T(rng.uniform(-1, 1, (11008, 4096)).astype(np.float32)))["id"]
    bl = T(rng.uniform(-1, 1, 11008).astype(np.float32))
    put("linear +bias", best(lambda: o.add(o.matmul(xl, wt)["id"], bl)), 2.0 * 16 * 4096 * 11008, "tensor",
        "16 of 16384 output rows")
    for xs, ws, st, pd in (([2, 64, 56, 56], [64, 64, 3, 3], 1, 1), ([2, 3, 224, 224], [64, 3, 7, 7], 2, 3)):
        tag = f"{ws[2]}x{ws[3]} s{st}"
        xc, wc = T(rng.standard_normal(xs, dtype=np.float32)), T(rng.standard_normal(ws, dtype=np.float32))
        oh = (xs[2] + 2 * pd - ws[2]) // st + 1
        ys = [2, ws[0], oh, oh]
        gy = T(rng.standard_normal(ys, dtype=np.float32))
        fl = 2.0 * 2 * ws[0] * oh * oh * xs[1] * ws[2] * ws[3]
        put(f"conv2d fwd {tag}", best(lambda: o.conv2d(xc, wc, None, [st], [pd], [1], 1)), fl, "tensor",
            "2 of 128 images")
        put(f"conv2d dgrad {tag}", best(lambda: o.conv2dInputBackward(gy, wc, xs, ys, [st], [pd])), fl, "tensor",
            "2 of 128 images")
        put(f"conv2d wgrad {tag}", best(lambda: o.conv2dWeightBackward(gy, xc, ws, ys, xs, [st], [pd])), fl, "tensor",
            "2 of 128 images")
        for h in (xc, wc, gy):
            o.destroy(h)
    # element-wise rows, full size
    xa = T(rng.standard_normal((16384, 11008), dtype=np.float32))
    ba = T(rng.standard_normal(11008, dtype=np.float32))
    put("add broadcast [M,N]+[N]", best(lambda: o.add(xa, ba)), 2 * 16384 * 11008 * 4 + 11008 * 4, "hbm")
    xb = T(rng.standard_normal((16384, 11008), dtype=np.float32))
    put("mul same-shape", best(lambda: o.mul(xa, xb)), 3 * 16384 * 11008 * 4, "hbm")
    for h in (xa, ba, xb):
        o.destroy(h)
    # multi-tensor optimizer rows on the first 8 of the 64 tensors (the oracle's
    # per-element loop has the same cost per element on every tensor); the same
    # hyper-parameters and bytes per element as the GPU rows
    sample = 8
    shp = [SHAPES[i % 4] for i in range(sample)]
    P = [T(rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for s in shp]
    G = [T(rng.standard_normal(s, dtype=np.float32) * np.float32(1e-3)) for s in shp]
    S0 = [T(np.zeros(s, np.float32)) for s in shp]
    S1 = [T(np.zeros(s, np.float32)) for s in shp]
    el = sum(numel(s) for s in shp)
    tag = f"{sample} of {NTENSORS} tensors ({el} of the elements)"
    ss, isb = adam_scalars(1)
    for name, bpe, fn in (
            ("sgd momentum 0.9 nesterov (multi-tensor)", 20,
             lambda: o.sgdStepMulti(P, G, S0, 1e-3, 0.9, 0.0, 0.0, True)),
            ("adam L2 wd (multi-tensor)", 28, lambda: o.adamStepMulti(P, G, S0, S1, LR, B1, B2, EPS, WD, ss, isb)),
            ("rmsprop momentum 0.9 (multi-tensor)", 28,
             lambda: o.rmspropStepMulti(P, G, S0, S1, 0.01, 0.99, 1e-8, 0.0, 0.9)),
            ("adagrad (multi-tensor)", 20, lambda: o.adagradStepMulti(P, G, S0, 0.01, 1e-10, 0.0)),
            ("adamax (multi-tensor)", 28,
             lambda: o.adamaxStepMulti(P, G, S0, S1, 0.002, 0.9, 0.999, 1e-8, 0.0, 0.02, 1.0)),
            ("nadam (multi-tensor)", 28, lambda: o.nadamStepMulti(P, G, S0, S1, 0.002, 0.9, 0.999, 1e-8, 0.0, 0.02, 0.9)),
            ("radam (multi-tensor)", 28,
             lambda: o.radamStepMulti(P, G, S0, S1, 1e-3, 0.9, 0.999, 1e-8, 0.0, 0.01, 0.53, 0.994, 6))):
        put(name, best(fn), bpe * el, "hbm", tag)
    for h in P + G + S0 + S1:
        o.destroy(h)
    return res


def run_ops(args):
    """Per-op throughput of the reductions / norms, the dense contractions and
    the multi-tensor SGD / Adam steps through the reference-facing runtime surface
    (CudaRuntime, handle API, outputs allocated per call from the pool), each
    against its roofline: HBM for the reductions and norms (algorithmic bytes:
    every input read once, every output written once), the 3xTF32 tensor rate
    for the contractions.  Inputs ~N(0,1) / ~U(-1,1) from the device RNG,
    larger than L2.  One JSON line with a result per op."""
    import torch
    from tpcuda import CudaRuntime
    rt = CudaRuntime(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.ExternalStream(rt.stream())
    hbm, _ = measured_peaks()
    peak3, bf16, peak_kind = tf32x3_peak()
    reps = max(3, min(args.steps, 10))
    rt.setSeed(0)
    results = []

    try:
        import pynvml
        pynvml.nvmlInit()
        nvml_dev = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
    except Exception:  # noqa: BLE001 - no NVML: rows carry no clock
        pynvml, nvml_dev = None, None
    last_clk = {}

    def read_clock():
        if nvml_dev is None:
            return {}
        try:
            r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(nvml_dev)
            return {"sm_mhz_end": pynvml.nvmlDeviceGetClockInfo(nvml_dev, pynvml.NVML_CLOCK_SM),
                    "sw_power_cap_end": bool(r & pynvml.nvmlClocksEventReasonSwPowerCap)}
        except Exception:  # noqa: BLE001
            return {}

    def timed(fn, n_out, idle=False):
        # outputs are destroyed as soon as they are made (stream-ordered), so the
        # pool serves every rep from the blocks of the warm-up call.  idle: a
        # contraction row starts after 0.25 s without GPU work, so it is timed in
        # the burst regime of the burst GEMM peak it is divided by, not under the
        # power cap that the previous rows' seconds of tensor work engage
        if idle:
            rt.synchronize()
            time.sleep(0.25)
        for _ in range(2):
            for o in fn()[:n_out]:
                rt.destroy(o["id"])
        rt.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            for o in fn()[:n_out]:
                rt.destroy(o["id"])
        e1.record(stream)
        e1.synchronize()
        last_clk.clear()
        last_clk.update(read_clock())
        return e0.elapsed_time(e1) / reps

    def add(name, shape, ms, work, bound):
        if bound == "hbm":
            achieved = work / (ms * 1e-3) / 1e9
            results.append({"op": name, "shape": shape, "ms": round(ms, 4), "GB/s": round(achieved, 1),
                            "frac_of_hbm": round(achieved / hbm, 3)})
        else:
            achieved = work / (ms * 1e-3) / 1e12
            results.append({"op": name, "shape": shape, "ms": round(ms, 4), "TFLOP/s": round(achieved, 2),
                            "frac_of_3xtf32": round(achieved / peak3, 3)})
        results[-1].update(last_clk)

    one = lambda h: [h]  # noqa: E731
    # ---- reductions and norms ----
    x = rt.randn([16384, 4096], "float32")
    g = rt.full([4096], 1.0, "float32")
    b = rt.full([4096], 0.0, "float32")
    dy = rt.randn([16384, 4096], "float32")
    nb = 16384 * 4096 * 4
    ms = timed(lambda: rt.layerNormForward(x["id"], [4096], g["id"], b["id"], 1e-5), 3)
    add("layer_norm fwd", [16384, 4096], ms, 2 * nb, "hbm")
    y, sm, sr = rt.layerNormForward(x["id"], [4096], g["id"], b["id"], 1e-5)
    ms = timed(lambda: rt.layerNormBackward(dy["id"], x["id"], [4096], g["id"], sm["id"], sr["id"]), 3)
    add("layer_norm bwd", [16384, 4096], ms, 3 * nb, "hbm")
    for h in (y, sm, sr, x, g, b, dy):
        rt.destroy(h["id"])
    x = rt.randn([32768, 8192], "float32")
    nb = 32768 * 8192 * 4
    add("softmax", [32768, 8192], timed(lambda: one(rt.softmax(x["id"], -1)), 1), 2 * nb, "hbm")
    add("log_softmax", [32768, 8192], timed(lambda: one(rt.logSoftmax(x["id"], -1)), 1), 2 * nb, "hbm")
    # backward: read the upstream gradient and the forward output, write the input gradient
    sm_out = rt.softmax(x["id"], -1)
    gy = rt.randn([32768, 8192], "float32")
    add("softmax bwd", [32768, 8192], timed(lambda: one(rt.softmaxBackward(gy["id"], sm_out["id"], 32768, 8192)), 1),
        3 * nb, "hbm")
    add("log_softmax bwd", [32768, 8192],
        timed(lambda: one(rt.logSoftmaxBackward(gy["id"], sm_out["id"], 32768, 8192)), 1), 3 * nb, "hbm")
    for h in (sm_out, gy):
        rt.destroy(h["id"])
    rt.destroy(x["id"])
    # element-wise chain with a zero-stride broadcast (the linear layer's bias add)
    xa = rt.randn([16384, 11008], "float32")
    ba = rt.randn([11008], "float32")
    add("add broadcast [M,N]+[N]", [16384, 11008], timed(lambda: one(rt.add(xa["id"], ba["id"])), 1),
        2 * 16384 * 11008 * 4 + 11008 * 4, "hbm")
    xb = rt.randn([16384, 11008], "float32")
    add("mul same-shape", [16384, 11008], timed(lambda: one(rt.mul(xa["id"], xb["id"])), 1),
        3 * 16384 * 11008 * 4, "hbm")
    for h in (xa, xb, ba):
        rt.destroy(h["id"])
    x = rt.randn([8192, 8192], "float32")
    nb = 8192 * 8192 * 4
    add("sum all", [8192, 8192], timed(lambda: one(rt.sum(x["id"])), 1), nb, "hbm")
    for d in (0, -1):
        add(f"sum dim {d}", [8192, 8192], timed(lambda: one(rt.sumDim(x["id"], d, False)), 1), nb, "hbm")
        add(f"mean dim {d}", [8192, 8192], timed(lambda: one(rt.meanDim(x["id"], d, False)), 1), nb, "hbm")
        add(f"max dim {d}", [8192, 8192], timed(lambda: rt.maxDim(x["id"], d, False), 2), nb, "hbm")
    rt.destroy(x["id"])
    shp = [256, 128, 56, 56]
    x = rt.randn(shp, "float32")
    dy = rt.randn(shp, "float32")
    g = rt.full([128], 1.0, "float32")
    b = rt.full([128], 0.0, "float32")
    rm = rt.full([128], 0.0, "float32")
    rv = rt.full([128], 1.0, "float32")
    nb = 256 * 128 * 56 * 56 * 4
    ms = timed(lambda: rt.batchNormTrain(x["id"], g["id"], b["id"], rm["id"], rv["id"], 1e-5, 0.1), 3)
    add("batch_norm train fwd", shp, ms, 2 * nb, "hbm")
    y, mean, inv = rt.batchNormTrain(x["id"], g["id"], b["id"], rm["id"], rv["id"], 1e-5, 0.1)
    ms = timed(lambda: rt.batchNormBackward(dy["id"], x["id"], g["id"], mean["id"], inv["id"]), 3)
    add("batch_norm bwd", shp, ms, 3 * nb, "hbm")
    for h in (y, mean, inv, x, dy, g, b, rm, rv):
        rt.destroy(h["id"])
    # ---- dense contractions ----
    for n in (512, 2048, 8192):
        a = rt.rand([n, n], "float32")
        bb = rt.rand([n, n], "float32")
        add("matmul", [n, n, n], timed(lambda: one(rt.matmul(a["id"], bb["id"])), 1, True), 2.0 * n ** 3, "tensor")
        rt.destroy(a["id"])
        rt.destroy(bb["id"])
    xl = rt.rand([16384, 4096], "float32")
    wl = rt.rand([11008, 4096], "float32")
    bl = rt.rand([11008], "float32")
    add("linear +bias", [16384, 4096, 11008], timed(lambda: one(rt.linear(xl["id"], wl["id"], bl["id"])), 1, True),
        2.0 * 16384 * 4096 * 11008, "tensor")
    for h in (xl, wl, bl):
        rt.destroy(h["id"])
    for xs, ws, st, pd in (([128, 64, 56, 56], [64, 64, 3, 3], 1, 1), ([128, 3, 224, 224], [64, 3, 7, 7], 2, 3)):
        xc = rt.randn(xs, "float32")
        wc = rt.randn(ws, "float32")
        oh = (xs[2] + 2 * pd - ws[2]) // st + 1
        ys = [xs[0], ws[0], oh, oh]
        gy = rt.randn(ys, "float32")
        fl = 2.0 * ys[0] * ys[1] * oh * oh * xs[1] * ws[2] * ws[3]
        tag = f"{ws[2]}x{ws[3]} s{st}"
        add(f"conv2d fwd {tag}", xs,
            timed(lambda: one(rt.conv2d(xc["id"], wc["id"], None, [st], [pd], [1], 1)), 1, True), fl, "tensor")
        add(f"conv2d dgrad {tag}", xs,
            timed(lambda: one(rt.conv2dInputBackward(gy["id"], wc["id"], xs, ys, [st], [pd])), 1, True), fl,
            "tensor")
        add(f"conv2d wgrad {tag}", xs,
            timed(lambda: one(rt.conv2dWeightBackward(gy["id"], xc["id"], ws, ys, xs, [st], [pd])), 1, True), fl,
            "tensor")
        for h in (xc, wc, gy):
            rt.destroy(h["id"])
    # ---- multi-tensor optimizer steps over the 64-tensor set (402.7 M elements) ----
    # (AdamW is the default workload's kernel; here the handle-API entries the
    # reference optimizers call: SGD momentum 0.9 nesterov, and Adam with L2 decay)
    rt.setSeed(1000)
    P = [rt.normal(SHAPES[i % 4], "float32", 0.0, 0.02) for i in range(NTENSORS)]
    G = [rt.normal(SHAPES[i % 4], "float32", 0.0, 1e-3) for i in range(NTENSORS)]
    S0 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(NTENSORS)]
    S1 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(NTENSORS)]
    elems = sum(numel(h["shape"]) for h in P)
    ids = lambda hs: [h["id"] for h in hs]  # noqa: E731

    def timed_inplace(fn):
        for _ in range(3):
            fn()
        rt.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    ms = timed_inplace(lambda: rt.sgdStepMulti(ids(P), ids(G), ids(S0), 1e-3, 0.9, 0.0, 0.0, True))
    add("sgd momentum 0.9 nesterov (multi-tensor)", [NTENSORS, elems], ms, 20 * elems, "hbm")
    ss, isb = adam_scalars(1)
    ms = timed_inplace(lambda: rt.adamStepMulti(ids(P), ids(G), ids(S0), ids(S1), LR, B1, B2, EPS, WD, ss, isb))
    add("adam L2 wd (multi-tensor)", [NTENSORS, elems], ms, 28 * elems, "hbm")
    # the other fused steps (rmsprop_step.wgsl, extended_step.wgsl) over the same set:
    # bytes per element read + written (Adagrad keeps one state tensor)
    ext = [("rmsprop momentum 0.9 (multi-tensor)", 28,
            lambda: rt.rmspropStepMulti(ids(P), ids(G), ids(S0), ids(S1), 0.01, 0.99, 1e-8, 0.0, 0.9)),
           ("adagrad (multi-tensor)", 20, lambda: rt.adagradStepMulti(ids(P), ids(G), ids(S0), 0.01, 1e-10, 0.0)),
           ("adamax (multi-tensor)", 28,
            lambda: rt.adamaxStepMulti(ids(P), ids(G), ids(S0), ids(S1), 0.002, 0.9, 0.999, 1e-8, 0.0, 0.02, 1.0)),
           ("nadam (multi-tensor)", 28,
            lambda: rt.nadamStepMulti(ids(P), ids(G), ids(S0), ids(S1), 0.002, 0.9, 0.999, 1e-8, 0.0, 0.02, 0.9)),
           ("radam (multi-tensor)", 28,
            lambda: rt.radamStepMulti(ids(P), ids(G), ids(S0), ids(S1), 1e-3, 0.9, 0.999, 1e-8, 0.0, 0.01, 0.53, 0.994,
                                      6))]
    for name, bpe, fn in ext:
        add(name, [NTENSORS, elems], timed_inplace(fn), bpe * elems, "hbm")
    for h in P + G + S0 + S1:
        rt.destroy(h["id"])
    cpu_cores = None
    if not args.no_cpu_baseline:
        os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
        cpu_cores = int(os.environ["OMP_NUM_THREADS"])
        cpu = cpu_ops()
        for r in results:
            key = f"matmul {r['shape'][0]}" if r["op"] == "matmul" else r["op"]
            if key in cpu:
                r["cpu_baseline"] = dict(cpu[key], kind="port", cores=cpu_cores)
    print(json.dumps({"metric": "per-op throughput vs roofline (reductions/norms/optimizers: GB/s of HBM; "
                                "contractions: TFLOP/s of 3xTF32)", "n_gpus": 1, "reps": reps, "hbm_peak_gbs": hbm,
                      "tf32x3_peak_tflops": round(peak3, 1), "peak_source": f"{peak_kind} bf16 {bf16}",
                      "path": "CudaRuntime handle API (the reference-facing surface), NCHW",
                      "timing": ("CUDA events over the reps after 2 warm-up calls; contraction rows start after "
                                 "0.25 s idle (burst regime, as the burst bf16 peak); sm_mhz_end: NVML SM clock "
                                 "right after each row's timed region"),
                      "cpu_baseline_cores": cpu_cores, "results": results}), flush=True)


TINY_TRACE = os.path.join(ROOT, "tests", "golden", "traces", "tiny_cnn.json")
TRACE_ID_BASE = 1_000_000_000


def replay_trace(rt, calls):
    """Issue a recorded runtime-call stream on ``rt`` (tensor ids remapped).

    Returns (wall time of each training step in s, largest deviation of any
    ``toList`` result from the recorded one relative to its scale).  A step
    starts at the bias readback before every second ``conv2d`` (the reference's
    conv2d takes its bias as a host list) and ends with the loss readback, so
    each step ends on a host sync and wall time is its duration."""
    conv = [i for i, c in enumerate(calls) if c["m"] == "conv2d"]
    starts = [conv[k] - 1 for k in range(0, len(conv), 2)]
    assert all(calls[i]["m"] == "toList" for i in starts) and calls[-1]["m"] == "toList"
    ids: dict[int, int] = {}

    def remap(v):
        if isinstance(v, bool):
            return v
        if isinstance(v, int) and v >= TRACE_ID_BASE:
            return ids[v]
        if isinstance(v, list):
            return [remap(x) for x in v]
        return v

    def learn(rec, res):
        if isinstance(rec, dict) and "id" in rec:
            ids[rec["id"]] = res["id"]
        elif isinstance(rec, list) and rec and isinstance(rec[0], dict):
            for r, q in zip(rec, res):
                learn(r, q)

    bounds = set(starts)
    marks, dev = [], 0.0
    for i, c in enumerate(calls):
        if i in bounds:
            marks.append(time.perf_counter())
        res = getattr(rt, c["m"])(*remap(c["a"]))
        if c["m"] == "toList":
            want = [float(v) for v in c["r"]]
            if want:
                scale = max(1.0, max(abs(v) for v in want))
                dev = max(dev, max(abs(a - float(b)) for a, b in zip(want, res)) / scale)
        else:
            learn(c["r"], res)
    marks.append(time.perf_counter())
    return [b - a for a, b in zip(marks, marks[1:])], dev


def run_tiny(args):
    """The Tiny-CNN training step (batch 64, 1x28x28 -> conv 1->8 -> pool ->
    conv 8->16 -> pool -> linear 784->10, Adam) as the reference package issues
    it: the runtime-call stream the unmodified reference ``torch`` package made
    for 10 training steps (tests/golden/traces/tiny_cnn.json), replayed on
    CudaRuntime, the reference-facing surface.  Latency-bound (37 MFLOP per
    forward): the metric is wall-clock ms per step, host readbacks included
    (the reference reads the conv bias back each call and the loss each step).
    The trace is replayed 1 + --steps//10 times (the first untimed); the same
    replay on the CPU oracle runtime is the CPU baseline."""
    import torch
    from tpcuda import CudaRuntime
    from tpcuda._lib import check
    import ctypes
    calls = json.load(open(TINY_TRACE))["calls"]
    rt = CudaRuntime(0)
    torch.cuda.set_device(0)
    reps = max(1, args.steps // 10)
    for _ in range(max(1, args.warmup // 10)):
        replay_trace(rt, calls)
    rt.synchronize()
    l0 = ctypes.c_int64(0)
    check(rt.lib.tp_kernel_launches(ctypes.byref(l0)))
    steps, dev = [], 0.0
    for _ in range(reps):
        t, d = replay_trace(rt, calls)
        steps += t
        dev = max(dev, d)
    l1 = ctypes.c_int64(0)
    check(rt.lib.tp_kernel_launches(ctypes.byref(l1)))
    ms = statistics.median(steps) * 1e3
    line = {"metric": "Tiny CNN train step (replayed reference runtime-call stream)", "value": round(ms, 4),
            "unit": "ms/step", "n_gpus": 1, "steps": len(steps), "warmup": 10 * max(1, args.warmup // 10),
            "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "replicas only",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded device RNG, as recorded)",
            "config": {"workload": "Tiny CNN, batch 64, Adam lr 1e-3, 10 recorded steps per replay",
                       "path": "CudaRuntime handle API, calls as the reference package issued them"},
            "gpu_launches": int((l1.value - l0.value) / max(1, len(steps))),
            "max_rel_dev_from_recorded": dev, "bound": "latency (host round trips per step)"}
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle_runtime import OracleRuntime
        orc = OracleRuntime()
        replay_trace(orc, calls)
        t, _ = replay_trace(orc, calls)
        line["cpu_baseline"] = {"value": round(statistics.median(t) * 1e3, 4), "unit": "ms/step",
                                "cores": os.cpu_count(), "kind": "port",
                                "sample": "the same recorded 10-step stream on the oracle runtime"}
    print(json.dumps(line), flush=True)


def vgg_launch_list(args):
    """Profiling aid (1 GPU): two eager VGG-11-BN steps at --batch, printing
    the kernel-launch counts so an ncu launch list can select exactly the
    second step (-s <first> -c <per step>)."""
    import numpy as np
    from tpcuda import CudaRuntime
    from tpcuda.vgg import VGG11BN
    rt = CudaRuntime(0)
    B = args.batch
    m = VGG11BN(rt, B, seed=0)
    rng = np.random.default_rng(0)
    m._h2d(m.x, rng.standard_normal((B, 3, 32, 32)).astype(np.float32))
    m._h2d(m.y, rng.integers(0, 10, B).astype(np.float32))
    n0 = rt.kernelLaunches()
    m.step_eager()
    rt.synchronize()
    n1 = rt.kernelLaunches()
    m.step_eager()
    rt.synchronize()
    n2 = rt.kernelLaunches()
    print(json.dumps({"launch_list": "vgg11-bn eager step", "batch": B, "launches_before_step2": n1 - n0,
                      "launches_per_step": n2 - n1, "loss": m.read_loss()}), flush=True)
    m.close()


def profile_case(args):
    """Profiling aid (1 GPU, no timing): two identical iterations of one per-op
    case on the handle API, so an ncu capture can select the second one.
      bn     BatchNorm2d train fwd + bwd on [256,128,56,56] (4 kernels per
             iteration: statistics, normalise, backward sums, backward apply)
      stem   the 7x7 stride-2 3 -> 64 convolution forward on [32,3,224,224]
             (one tensor-core GEMM per iteration)
      optim  RMSprop (momentum 0.9) then NAdam over 8 tensors of the optimizer
             workload's shapes (one fused launch each per iteration)"""
    from tpcuda import CudaRuntime
    rt = CudaRuntime(0)
    rt.setSeed(0)
    ids = lambda hs: [h["id"] for h in hs]  # noqa: E731
    if args.profile_case == "bn":
        shp = [256, 128, 56, 56]
        x, dy = rt.randn(shp, "float32"), rt.randn(shp, "float32")
        g, b = rt.full([128], 1.0, "float32"), rt.full([128], 0.0, "float32")
        rm, rv = rt.full([128], 0.0, "float32"), rt.full([128], 1.0, "float32")

        def it():
            y, mean, inv = rt.batchNormTrain(x["id"], g["id"], b["id"], rm["id"], rv["id"], 1e-5, 0.1)
            for h in [y, mean, inv] + rt.batchNormBackward(dy["id"], x["id"], g["id"], mean["id"], inv["id"]):
                rt.destroy(h["id"])
    elif args.profile_case == "stem":
        x, w = rt.randn([32, 3, 224, 224], "float32"), rt.randn([64, 3, 7, 7], "float32")

        def it():
            rt.destroy(rt.conv2d(x["id"], w["id"], None, [2], [3], [1], 1)["id"])
    else:
        P = [rt.normal(SHAPES[i % 4], "float32", 0.0, 0.02) for i in range(8)]
        G = [rt.normal(SHAPES[i % 4], "float32", 0.0, 1e-3) for i in range(8)]
        S0 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(8)]
        S1 = [rt.zeros(SHAPES[i % 4], "float32") for i in range(8)]

        def it():
            rt.rmspropStepMulti(ids(P), ids(G), ids(S0), ids(S1), 0.01, 0.99, 1e-8, 0.0, 0.9)
            rt.nadamStepMulti(ids(P), ids(G), ids(S0), ids(S1), 0.002, 0.9, 0.999, 1e-8, 0.0, 0.02, 0.9)
    for _ in range(2):
        it()
    rt.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "iterations": 2}), flush=True)


VGG_CONVS = ((64, 128, 16), (128, 256, 8), (256, 256, 8), (256, 512, 4), (512, 512, 4), (512, 512, 2))


def run_conv_layer(args):
    """One VGG-11-BN convolution pass on channels-last buffers with packed
    [Cout][3][3][Cin] filters (the step's own layout and entries), timed with
    CUDA events over --steps launches after --warmup; doubles as a small,
    few-launch target for ncu captures of one GEMM kernel.  One JSON line.
    --conv all: every tensor-core layer of the network (the 3x3 convolutions
    after the first), all three passes, one line each."""
    import torch
    from tpcuda import CudaRuntime
    rt = CudaRuntime(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.ExternalStream(rt.stream())
    if args.conv == "all":
        for cin, cout, hw in VGG_CONVS:
            for ps in ("fwd", "dgrad", "wgrad"):
                conv_pass(args, rt, stream, cin, cout, hw, ps)
    else:
        cin, cout, hw = (int(v) for v in args.conv.split(","))
        conv_pass(args, rt, stream, cin, cout, hw, args.pass_)


def conv_pass(args, rt, stream, cin, cout, hw, pass_):
    import ctypes
    import torch
    from tpcuda._lib import check
    lib = rt.lib
    B = args.batch
    check(lib.tp_set_gemm_path(args.gemm_path))
    rt.setSeed(0)
    hx = rt.randn([B, hw, hw, cin], "float32")
    fl = args.filter_layout
    hw_ = rt.randn([cout, 3, 3, cin] if fl else [cout, cin, 3, 3], "float32")
    hb = rt.randn([cout], "float32")
    hy = rt.randn([B, hw, hw, cout], "float32")
    hdx = rt.randn([B, hw, hw, cin], "float32")
    hdw = rt.randn([cout, 3, 3, cin], "float32")  # same size in either filter layout
    p = lambda h: ctypes.c_void_p(rt.devicePtr(h["id"]))  # noqa: E731
    x, w, b, y, dx, dw = (p(h) for h in (hx, hw_, hb, hy, hdx, hdw))
    if pass_ == "fwd":
        fn = lambda: lib.tpk_conv2d_fwd_nhwc(x, w, b, y, B, cin, hw, hw, cout, 3, 3, 1, 1, fl)  # noqa: E731
    elif pass_ == "dgrad":
        fn = lambda: lib.tpk_conv2d_dgrad_nhwc(y, w, dx, B, cin, hw, hw, cout, 3, 3, 1, 1, fl)  # noqa: E731
    else:
        fn = lambda: lib.tpk_conv2d_wgrad_nhwc(y, x, dw, B, cin, hw, hw, cout, 3, 3, 1, 1, fl)  # noqa: E731
    for _ in range(args.warmup):
        check(fn())
    rt.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        check(fn())
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    st = ctypes.c_int(0)
    check(lib.tp_gemm_status(ctypes.byref(st), 1))
    flops = 2.0 * B * hw * hw * cout * cin * 9
    peak3, _, peak_kind = tf32x3_peak()
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({"conv": [cin, cout, hw], "pass": pass_, "batch": B, "gemm_path": args.gemm_path,
                      "filter_layout": fl,
                      "ms": round(ms, 4), "TFLOP/s": round(tf, 2), "frac_of_3xtf32": round(tf / peak3, 3),
                      "peak": round(peak3, 1), "peak_source": peak_kind, "status": st.value}), flush=True)
    for h in (hx, hw_, hb, hy, hdx, hdw):
        rt.destroy(h["id"])


def run_vgg(args, rank, world, local):
    import ctypes

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    from tpcuda import CudaRuntime
    from tpcuda.dp import comm_from_store
    from tpcuda.vgg import VGG11BN
    rt = CudaRuntime(local)
    store = make_store(rank, world)
    stream = torch.cuda.ExternalStream(rt.stream(), device=torch.device("cuda", local))
    from tpcuda._lib import check as _check
    _check(rt.lib.tp_set_comm_priority(args.comm_priority))
    comm = comm_from_store(rt.lib, store)
    B = VGG_GLOBAL_BATCH // world
    model = VGG11BN(rt, B, seed=0, world=world, comm=comm)
    rng = np.random.default_rng(100 + rank)
    hx = torch.from_numpy(rng.standard_normal((B, 3, 32, 32)).astype(np.float32)).pin_memory()
    hy = torch.from_numpy(rng.integers(0, 10, B).astype(np.float32)).pin_memory()
    model.set_batch_device(hx.data_ptr(), hy.data_ptr())
    model.capture()
    for _ in range(args.warmup):
        model.step()
    rt.synchronize()

    def barrier():
        rt.synchronize()
        store.barrier()

    # ---- device-resident timed region: graph replays of the whole step ----
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    launches0 = rt.kernelLaunches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        model.step()
    e1.record(stream)
    e1.synchronize()
    launches = rt.kernelLaunches() - launches0
    clk = clocks.stop()
    ms_step = store.max(e0.elapsed_time(e1)) / args.steps
    value = VGG_GLOBAL_BATCH / (ms_step * 1e-3)
    loss_after = model.read_loss()

    # ---- end to end: pinned host batch -> HBM, step, loss back to host ----
    e2e_steps = max(3, min(args.steps, 20))
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        model.set_batch_device(hx.data_ptr(), hy.data_ptr())
        model.step()
        model.read_loss()
    f1.record(stream)
    f1.synchronize()
    e2e_ms = store.max(f0.elapsed_time(f1)) / e2e_steps
    e2e_value = VGG_GLOBAL_BATCH / (e2e_ms * 1e-3)

    # ---- dominant kernel: the implicit-GEMM convolution of block 4 (256->256 @ 8x8),
    # timed alone with events on the library stream ----
    b4 = model.blocks[3]
    lib = rt.lib
    flops = 2.0 * B * b4["cout"] * b4["H"] * b4["W"] * b4["cin"] * 9
    reps = 20
    xin = model.blocks[2]["out"]
    conv_args = (ctypes.c_void_p(xin), ctypes.c_void_p(model.p("conv3.w")), ctypes.c_void_p(model.p("conv3.b")),
                 ctypes.c_void_p(b4["z"]), B, b4["cin"], b4["H"], b4["W"], b4["cout"], 3, 3)
    if model.layout == "nhwc":
        conv_fn, conv_args = lib.tpk_conv2d_fwd_nhwc, conv_args + (1, 1, model.filter_layout(3))
    else:
        conv_fn, conv_args = lib.tpk_conv2d_fwd, conv_args + (1, 1, 1, 1)
    conv_fn(*conv_args)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(reps):
        conv_fn(*conv_args)
    g1.record(stream)
    g1.synchronize()
    k_ms = g0.elapsed_time(g1) / reps
    achieved = flops / (k_ms * 1e-3) / 1e12
    peak3, bf16, peak_kind = tf32x3_peak()
    hbm_peak, _ = measured_peaks()
    sm_mhz_max = float((clk or {}).get("sm_max_mhz") or 1965.0)
    n_sm = torch.cuda.get_device_properties(local).multi_processor_count
    cuda_peak = n_sm * 128 * 2 * sm_mhz_max * 1e6 / 1e12
    sr = model.step_roofline_ms(peak3, cuda_peak, hbm_peak)
    gemm_status = ctypes.c_int(0)
    lib.tp_gemm_status(ctypes.byref(gemm_status), 1)

    if comm is not None:
        comm.sync(60000)
    model.close()
    if comm is not None:
        comm.close()
    del hx, hy
    barrier()

    # ---- the fused AdamW step (the metric's other half), on one GPU ----
    adamw = None
    if world == 1 and not args.no_adamw:
        adamw = measure_adamw(args, rt, rank, world, store, args.tensors)
    store.close()
    if rank != 0:
        return
    line = {
        "metric": "VGG-11-BN train imgs/s", "value": round(value, 1), "unit": "imgs/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": VGG_WORKLOAD, "global_batch": VGG_GLOBAL_BATCH, "per_rank_batch": B,
                   "parallelism": f"dp{world}", "l2": "per-step activations ~1.6 GB per rank at batch 1024 > L2",
                   "loss_after_timed_steps": round(loss_after, 5),
                   "collective": "bucketed NCCL all-reduce of the gradients, overlapped with backward" if world > 1
                   else "none (one rank)"},
        "gpu_launches": int(launches),
        "clocks": clk,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak3, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak3, 4), "traffic": None,
                     "peak_source": f"{peak_kind} bf16_tflops {bf16} / 2 (tf32) / 3 (3xTF32)",
                     "kernel": ("conv3x3 forward, TMA-fed tcgen05 implicit GEMM, channels-last"
                                if model.layout == "nhwc" else "conv3x3 forward, gather-GEMM, NCHW")
                     + ", block 4 (256->256 @ 8x8)",
                     "kernel_ms": round(k_ms, 4), "step_tflops": round(model.step_flops() * world / 1e12, 4),
                     "gemm_status": gemm_status.value},
        "e2e": {"value": round(e2e_value, 1), "unit": "imgs/s",
                "h2d_bytes_per_step": int(VGG_GLOBAL_BATCH * (3 * 32 * 32 + 1) * 4),
                "d2h_bytes_per_step": 4 * world,
                "path": "per rank: tp_memcpy_h2d(pinned batch) + tp_graph_launch(step) + loss readback"},
        "step_roofline": {"min_ms": round(sr["min_ms"], 4), "frac": round(sr["min_ms"] / ms_step, 4),
                          "tensor_ms": round(sr["tensor_ms"], 4), "cuda_core_ms": round(sr["cuda_core_ms"], 4),
                          "hbm_ms": round(sr["hbm_ms"], 4), "hbm_gb": round(sr["hbm_bytes"] / 1e9, 3),
                          "basis": (f"per-rank step: contractions at the 3xTF32 peak {round(peak3, 1)} TFLOP/s, the "
                                    f"first layer at the CUDA-core fp32 peak {round(cuda_peak, 1)} TFLOP/s "
                                    f"({n_sm} SMs x 128 lanes x 2 x max SM clock), BatchNorm / pool / SGD bytes at "
                                    f"the measured HBM {hbm_peak} GB/s")},
    }
    # DRAM traffic of the dominant kernel from one ncu capture at batch 1024
    # (profiles/), scaled by the per-rank batch
    tf = os.path.join(ROOT, "profiles", "conv3x3_tma2_pair_fwd_256to256_8x8_b1024_traffic.json")
    if os.path.exists(tf) and model.layout == "nhwc":
        t = json.load(open(tf))
        line["roofline"]["traffic"] = int(t["bytes_per_launch"] * B / t["batch"])
    if world == 1 and not args.no_cpu_baseline:
        os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
        r = cpu_vgg(VGG_CPU_BATCH, 3)
        line["cpu_baseline"] = {"value": round(r["imgs_per_s"], 4), "unit": "imgs/s",
                                "cores": int(os.environ["OMP_NUM_THREADS"]), "kind": "port",
                                "sample": f"oracle composition of the same step at batch {VGG_CPU_BATCH} (model "
                                          f"resident, SGD each step), median of 3 steps after 1 warm-up"}
    if adamw is not None:
        if not args.no_cpu_baseline:
            adamw["cpu_baseline"] = adamw_cpu_baseline()
        line["adamw"] = adamw
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["vgg", "adamw", "ops", "conv", "tiny"], default="vgg")
    ap.add_argument("--conv", default="256,256,8",
                    help="--workload conv: Cin,Cout,H=W of the layer, or 'all' (every tensor-core layer, 3 passes)")
    ap.add_argument("--pass", dest="pass_", choices=["fwd", "dgrad", "wgrad"], default="fwd",
                    help="--workload conv: which pass")
    ap.add_argument("--gemm-path", type=int, default=0, help="--workload conv: tp_set_gemm_path value")
    ap.add_argument("--filter-layout", type=int, default=1,
                    help="--workload conv: 1 = [Cout][3][3][Cin] (the step's), 0 = [Cout][Cin][3][3] (with Cin = 4: "
                         "the first layer's CUDA-core kernels)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--comm-priority", type=int, choices=[0, 1], default=1,
                    help="vgg workload at N>1: 1 = the communicator's stream at the highest priority (the "
                         "default), 0 = normal priority")
    ap.add_argument("--no-adamw", action="store_true", help="vgg workload at N=1: skip the fused AdamW sub-record")
    ap.add_argument("--launch-list", action="store_true",
                    help="profiling aid: two eager VGG steps at --batch with launch counts (1 GPU, no timing)")
    ap.add_argument("--batch", type=int, default=VGG_GLOBAL_BATCH, help="per-GPU batch for --launch-list")
    ap.add_argument("--tensors", type=int, default=NTENSORS,
                    help="number of parameter tensors (64 = the benchmark; fewer for profiler captures)")
    ap.add_argument("--profile-case", choices=["bn", "stem", "optim"], default=None,
                    help="profiling aid: two iterations of one per-op case (1 GPU, no timing)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        profile_case(args)
        return
    if args.launch_list:
        vgg_launch_list(args)
        return
    if args.workload == "ops" and args.impl == "ours":
        run_ops(args)
        return
    if args.workload == "conv" and args.impl == "ours":
        run_conv_layer(args)
        return
    if args.workload == "tiny" and args.impl == "ours":
        run_tiny(args)
        return
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload == "vgg":
        run_vgg(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
