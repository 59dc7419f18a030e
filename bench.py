"""Benchmark of the compiled-plan training step on B200 (one process per GPU).

``python bench.py --gpus N --steps K --warmup W [--config charmlp|gpt2|mlp|fused|gemm|gemm_skinny]
[--impl reference]`` prints ONE JSON line on rank 0.

A step is one run of the recorded-gradient training plan (loss and every
gradient), the gradient all-reduce across ranks (N > 1) and the optimizer
update, replayed as one CUDA graph.  ``value`` is whole-job samples/s timed on
the device with inputs resident in HBM; ``e2e`` is the same metric through the
public API with the step's inputs copied from pinned host memory and the loss
read back every step.  ``--impl reference`` times the reference interpreter's
arithmetic (the C++ restatement in ``oracle/``, the reference itself being Rust
that cannot be built here) on the host cores for the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DEFAULT_CONFIG = "charmlp"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 6:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(sm)}


def dist_setup(gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


CONFIGS = {
    "charmlp": (lambda: __import__("poorgrad_b200.configs").configs.char_mlp(batch=16384, seed=4),
                {"model": "char-mlp-lm", "global_batch_per_gpu": 16384, "context": 8,
                 "embedding": 64, "hidden": 512, "vocab": 27}),
    "gpt2": (lambda: __import__("poorgrad_b200.configs").configs.gpt2(),
             {"model": "gpt2-small-shaped", "global_batch_per_gpu": 8, "seq_len": 1024,
              "layers": 12, "d_model": 768}),
    "mlp": (lambda: __import__("poorgrad_b200.configs").configs.mlp(batch=128),
            {"model": "mlp-784-256-10", "global_batch_per_gpu": 128}),
    "fused": (lambda: __import__("poorgrad_b200.configs").configs.fused(),
              {"model": "fused-8192x8192"}),
    "gemm": (lambda: __import__("poorgrad_b200.configs").configs.gemm(),
             {"model": "gemm-4096^3-fwd+bwd"}),
    "gemm_skinny": (lambda: __import__("poorgrad_b200.configs").configs.gemm(32768, 768, 3072),
                    {"model": "gemm-32768x768x3072-fwd+bwd"}),
}


def build_workload(name: str, rank: int, config_only: bool = False):
    make, cfg = CONFIGS[name]
    return (None if config_only else make()), dict(cfg)


def reference_arm(args, name):
    """Times the reference interpreter's arithmetic (the oracle port) on the
    host cores: shards of a bounded sample, one per core, run concurrently."""
    rank, world, local = dist_setup(args.gpus)
    if rank != 0:
        return
    import oracle
    from poorgrad_b200 import configs
    cores = os.cpu_count() or 1
    shard = {"charmlp": 64, "mlp": 128, "gpt2": None, "fused": None, "gemm": None,
             "gemm_skinny": None}[name]
    if name == "gpt2":
        w = configs.gpt2(batch=1, seq=128)
        unit_scale = 1.0  # one short sequence per shard
        sample = "1 sequence of 128 tokens per core (full 12-layer GPT-2-small widths)"
    elif name in ("fused", "gemm", "gemm_skinny"):
        w = {"fused": lambda: configs.fused(rows=256, cols=8192),
             "gemm": lambda: configs.gemm(256, 4096, 4096),
             "gemm_skinny": lambda: configs.gemm(256, 768, 3072)}[name]()
        sample = "256-row slice of the workload per core"
        unit_scale = 1.0
    else:
        w = configs.char_mlp(batch=shard) if name == "charmlp" else configs.mlp(batch=shard)
        sample = f"batch {shard} of the same graph per core"
    oracle.build()
    params = w.network.parameters()
    feeds = [w.feeds(i) for i in range(cores)]

    def one_step():
        threads = [threading.Thread(target=oracle.run, args=(w.columns, params, feeds[i]))
                   for i in range(cores)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()

    for _ in range(max(1, min(args.warmup, 1))):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = (time.perf_counter() - t0) / args.steps
    if name == "gpt2":
        value = cores * 1 / dt
        unit = "sequences/s"
    elif name == "fused":
        value = cores * 256 / dt
        unit = "rows/s"
    elif name in ("gemm", "gemm_skinny"):
        value = cores * 256 / dt
        unit = "rows/s"
    else:
        value = cores * shard / dt
        unit = "samples/s"
    _, cfg = build_workload(name, 0, config_only=True)
    cfg.update({"workload": name, "parallelism": f"dp{args.gpus}"})
    line = {"impl": "reference", "metric": "train samples/s" if unit == "samples/s" else f"train {unit}",
            "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded splitmix64 streams)",
            "config": cfg,
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(name):
    """The oracle on one host core, on a bounded sample of the same workload."""
    import oracle
    from poorgrad_b200 import configs
    oracle.build()
    if name == "gpt2":
        w = configs.gpt2(batch=1, seq=128)
        n, unit, sample = 1, "sequences/s", "1 sequence of 128 tokens, full model widths"
    elif name == "charmlp":
        w = configs.char_mlp(batch=256)
        n, unit, sample = 256, "samples/s", "batch 256 of the same graph, 1 step"
    elif name == "mlp":
        w = configs.mlp(batch=128)
        n, unit, sample = 128, "samples/s", "the full batch-128 step"
    else:
        return None
    params = w.network.parameters()
    feeds = w.feeds(0)
    oracle.run(w.columns, params, feeds)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < 10.0 or reps < 1:
        oracle.run(w.columns, params, feeds)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": n / dt, "unit": unit, "cores": 1, "kind": "port", "sample": sample}


KTYPES = ["ew", "row", "reduce", "prep", "gemm", "sort", "scatter", "fold", "final", "segsum"]


def kernel_profile(plan, reps=20):
    from poorgrad_b200.abi import load_library
    lib = load_library()
    lib.tbx_profile_kernels.restype = C.c_int64
    n = len(plan.describe().splitlines())
    ms = (C.c_float * n)()
    count = lib.tbx_profile_kernels(plan.handle, reps, ms, n)
    rows = []
    for k in range(max(0, count)):
        facts = (C.c_int64 * 8)()
        lib.tbx_kernel_facts(plan.handle, k, facts)
        rows.append({"k": k, "type": KTYPES[facts[0]], "ms": float(ms[k]), "batch": facts[1],
                     "m": facts[2], "n": facts[3], "kdim": facts[4], "read": facts[5],
                     "write": facts[6]})
    return rows


# DRAM read + write bytes per launch of the dominant kernel class, from one ncu
# launch-list capture of the workload (dram__bytes_read.sum +
# dram__bytes_write.sum; charmlp: its 63 k_gemm_tcgen05 launches average 77.3 MB).
NCU_TRAFFIC = {"charmlp": {"gemm": 77.29e6}}


def traffic(workload, kind):
    return NCU_TRAFFIC.get(workload, {}).get(kind)


def roofline(rows, workload=None):
    """Roofline of the dominant kernel: the kernel class with the largest share
    of the step (each GEMM launch is the same tcgen05 kernel).  achieved =
    algorithmic work of its launches / their summed device time; traffic = the
    ncu-measured DRAM bytes per launch of that class, where one was captured."""
    hbm, bf16, bf16_sus, how = peaks()
    total = sum(r["ms"] for r in rows) or 1.0
    by = {}
    for r in rows:
        by.setdefault(r["type"], []).append(r)
    kind, group = max(by.items(), key=lambda kv: sum(r["ms"] for r in kv[1]))
    t = sum(r["ms"] for r in group) * 1e-3
    if kind == "gemm":
        flops = sum(2.0 * r["batch"] * r["m"] * r["n"] * r["kdim"] for r in group)
        achieved = flops / t / 1e12
        peak = bf16 / 6.0   # tf32 runs at half the bf16 rate; 3xTF32 issues three products
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic(workload, kind),
                "traffic_unit": "bytes per launch", "launches": len(group),
                "kernel": "k_gemm_tcgen05 (3xTF32, all GEMMs of the step)",
                "share": t * 1e3 / total,
                "peak_note": f"3xTF32-effective = {how} bf16 {bf16:.0f} TF/s / 6"}
    bytes_ = sum(r["read"] + r["write"] for r in group)
    achieved = bytes_ / t / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "traffic": traffic(workload, kind),
            "traffic_unit": "bytes per launch", "launches": len(group),
            "kernel": f"{kind} kernels", "share": t * 1e3 / total,
            "peak_note": f"{how} HBM copy bandwidth"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200")
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-kernel-profile", action="store_true",
                    help="skip the per-kernel timing pass (for runs under a profiler)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args, args.config)

    import torch
    import torch.distributed as dist
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    from poorgrad_b200 import backend
    from poorgrad_b200.abi import Feeds, TbFeed
    code, msg = backend.status()
    if code != 0:
        raise SystemExit(f"backend unavailable: {code} {msg}")

    w, cfg = build_workload(args.config, rank)
    params = w.network.parameters()
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params)
    opt_cfg = w.optimizer
    opt = None
    if opt_cfg:
        kind = {"sgd": backend.SGD, "adam": backend.ADAM, "adamw": backend.ADAMW}[opt_cfg["kind"]]
        opt = backend.Optimizer(plan, dp, kind, zip(w.params, w.grads), opt_cfg["lr"],
                                opt_cfg.get("beta1", 0.9), opt_cfg.get("beta2", 0.999),
                                opt_cfg.get("eps", 1e-8), opt_cfg.get("decay", 0.0),
                                gradient_scale=1.0 / world)
    comm = None
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.tensor(list(backend.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = backend.Comm(rank, world, bytes(uid.cpu().tolist()))
        comm.attach(plan)

    # per-step batches: device-resident (value) and pinned host (e2e)
    nb = max(2, min(8, args.steps))
    host_batches = [w.feeds(1000 * rank + i) for i in range(nb)]
    sym_of = {}
    dev_bufs, pin_bufs = [], []
    for fb in host_batches:
        dfeed, pfeed = {}, {}
        for sym, payload in fb.items():
            if hasattr(payload, "indices"):
                arr = torch.from_numpy(np.ascontiguousarray(payload.indices, np.int32))
                kind = "indices"
            else:
                arr = torch.from_numpy(np.ascontiguousarray(payload.to_numpy(), np.float32))
                kind = "dense"
            d = arr.cuda()
            p = arr.pin_memory()
            dev_bufs.append(d)
            pin_bufs.append(p)
            dfeed[sym] = ("device", d.data_ptr(), kind)
            pfeed[sym] = ("host", p.data_ptr(), kind)
        sym_of[len(sym_of)] = (dfeed, pfeed)
    h2d = sum(b.numel() * b.element_size() for b in pin_bufs) // nb

    def step(i, host=False):
        feeds = sym_of[i % nb][1 if host else 0]
        plan.forward(dp, feeds)

    # warm-up (graph capture happens on the first run)
    for i in range(max(3, args.warmup)):
        step(i)
    plan.synchronize()
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(plan.stream())

    def timed(host):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        plan.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        loss_host = np.empty((), np.float32)
        t_wall = time.perf_counter()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(args.steps):
                step(i, host)
                if host:
                    loss_host = plan.of(w.loss)  # D2H of the step's loss (waits)
            end.record(stream)
        plan.synchronize()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
        wall = (time.perf_counter() - t_wall) * 1e3
        t = torch.tensor([ms], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(t.item()), wall, loss_host

    with Clocks(local) as clocks:
        ms, wall, _ = timed(False)
    ms_e2e, wall_e2e, last_loss = timed(True)
    per_step = ms / args.steps
    samples = w.samples * world
    value = samples / (per_step * 1e-3)
    e2e_value = samples / (ms_e2e / args.steps * 1e-3)

    stats = plan.stats()
    rows = kernel_profile(plan) if rank == 0 and not args.no_kernel_profile else []
    roof = roofline(rows, args.config) if rows else None
    if rank == 0:
        cpu = None if args.no_cpu else cpu_baseline(args.config)
        arena_mb = stats["arena_bytes"] / 2**20
        cfg.update({"workload": args.config, "parallelism": f"dp{world}",
                    "l2": f"working set > L2: arena {arena_mb:.0f} MiB per step, no flush",
                    "optimizer": opt_cfg.get("kind") if opt_cfg else None})
        line = {"metric": "train samples/s", "value": value, "unit": "samples/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded splitmix64 streams)",
                "config": cfg,
                "e2e": {"value": e2e_value, "unit": "samples/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": 4, "wall_ms": wall_e2e},
                "gpu_launches": stats["kernels"] * args.steps,
                "roofline": roof, "cpu_baseline": cpu, "clocks": clocks.summary(),
                "loss": float(last_loss), "wall_ms_timed": wall,
                "kernels_per_step": stats["kernels"], "gemms_per_step": stats["gemms"]}
        if os.environ.get("TB_PROFILE_OUT"):
            with open(os.environ["TB_PROFILE_OUT"], "w") as f:
                json.dump({"rows": rows, "describe": plan.describe()}, f, indent=1)
        print(json.dumps(line), flush=True)
    if world > 1:
        # leave without running destructors: tearing down communicators that
        # are still bound into a captured graph can block at interpreter exit
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
