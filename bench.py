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
    """Samples the SM clock and the throttle reasons of this process's GPU
    in-process through read-only NVML queries every ``period`` seconds, across
    the untimed replay and the timed region."""

    REASONS = [("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown")]

    def __init__(self, local: int, period: float = 0.005):
        self.local = local
        self.period = period
        self.samples = []       # (t, sm_mhz, reasons bitmask)
        self.stop = threading.Event()
        self.nvml = None
        self.handle = None
        self.max_mhz = None
        self.error = None
        self.marks = {}

    def __enter__(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.local).uuid)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.local)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception as e:  # no NVML: the line says so
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _run(self):
        n = self.nvml
        while not self.stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                why = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((time.perf_counter(), sm, why))
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
                return
            time.sleep(self.period)

    def mark(self, name):
        self.marks[name] = time.perf_counter()

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    "error": self.error}
        n = self.nvml
        t0 = self.marks.get("timed_start", 0.0)
        t1 = self.marks.get("timed_end", float("inf"))
        timed = [s for s in self.samples if t0 <= s[0] <= t1]
        names = sorted({name for _, _, why in self.samples for name, attr in self.REASONS
                        if why & getattr(n, attr, 0)})
        return {"sm_mhz": statistics.median(s[1] for s in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples), "samples_timed": len(timed),
                "sm_mhz_timed": statistics.median(s[1] for s in timed) if timed else None,
                "source": f"NVML in-process every {self.period * 1e3:.0f} ms over the untimed "
                          "replay and the timed steps"}


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


def build_workload(name: str, rank: int, config_only: bool = False, overrides=None):
    """The workload and its config; ``overrides`` (from --batch/--seq/--layers)
    resize charmlp, mlp and gpt2 for profiling captures, and say so in the
    config.  The default run uses none."""
    make, cfg = CONFIGS[name]
    cfg = dict(cfg)
    o = {k: v for k, v in (overrides or {}).items() if v}
    if o and name in ("charmlp", "mlp", "gpt2"):
        from poorgrad_b200 import configs
        if name == "charmlp":
            make = lambda: configs.char_mlp(batch=o.get("batch", 16384), seed=4)
        elif name == "mlp":
            make = lambda: configs.mlp(batch=o.get("batch", 128))
        else:
            make = lambda: configs.gpt2(batch=o.get("batch", 8), seq=o.get("seq", 1024),
                                        layers=o.get("layers", 12))
        cfg.update({"global_batch_per_gpu": o.get("batch", cfg.get("global_batch_per_gpu")),
                    "resized_for_profiling": o})
    return (None if config_only else make()), cfg


def metric_of(name):
    """(metric, unit, units per sample) of a config's line: GPT-2 counts
    tokens, the microbenches rows of their workload, the rest samples."""
    if name == "gpt2":
        return "train tokens/s", "tokens/s"
    if name in ("fused", "gemm", "gemm_skinny"):
        return "train rows/s", "rows/s"
    return "train samples/s", "samples/s"


def tree_sum(parts):
    """`tree_sum` of examples/makemore/mlp_parallel.rs:59-71: left + right in
    pairs, an odd last shard carried up."""
    while len(parts) > 1:
        nxt = [parts[i] + parts[i + 1] for i in range(0, len(parts) - 1, 2)]
        if len(parts) % 2:
            nxt.append(parts[-1])
        parts = nxt
    return parts[0]


def reference_arm(args, name):
    """Times the reference interpreter's arithmetic (the oracle port) on the
    host cores, in the reference's own data-parallel idiom
    (examples/makemore/mlp_parallel.rs): each step splits the workload's batch
    into one shard per core, runs the shards' plans on concurrent threads, sums
    the shard gradients in `tree_sum` order, scales by 1/shards and applies the
    config's optimizer on the host."""
    rank, world, local = dist_setup(args.gpus)
    if rank != 0:
        return
    import oracle
    from oracle import optim
    from poorgrad_b200 import configs
    cores = os.cpu_count() or 1
    metric, unit = metric_of(name)
    if name == "gpt2":
        # a full 8 x 1024 step would take the host cores many minutes: one
        # 128-token sequence per core at the full model widths
        w = configs.gpt2(batch=1, seq=128)
        per_shard, sample = 128, f"{cores} shards x 1 sequence of 128 tokens (full GPT-2-small widths) per step"
    elif name in ("fused", "gemm", "gemm_skinny"):
        w = {"fused": lambda: configs.fused(rows=256, cols=8192),
             "gemm": lambda: configs.gemm(256, 4096, 4096),
             "gemm_skinny": lambda: configs.gemm(256, 768, 3072)}[name]()
        per_shard, sample = 256, f"{cores} shards x a 256-row slice of the workload per step"
    else:
        full = 16384 if name == "charmlp" else 128
        per_shard = max(1, full // cores)
        w = (configs.char_mlp(batch=per_shard, seed=4) if name == "charmlp"
             else configs.mlp(batch=per_shard))
        sample = f"the full batch {per_shard * cores} as {cores} shards of {per_shard} per step"
    oracle.build()
    params = [p.reshape(w.columns.nodes[s.index].shape).copy()
              for p, s in zip(w.network.parameters(), w.params)]
    opt = w.optimizer
    host = optim.make(opt["kind"], opt) if opt else None
    results = [None] * cores

    def shard(i, feeds):
        results[i] = oracle.run(w.columns, params, feeds, read=[g.index for g in w.grads])

    def one_step(step):
        nonlocal params
        threads = [threading.Thread(target=shard, args=(i, w.feeds(step * cores + i)))
                   for i in range(cores)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if host is not None:
            grads = [tree_sum([results[i][g.index] for i in range(cores)]) * np.float32(1.0 / cores)
                     for g in w.grads]
            params = host.step(params, [g.astype(np.float32) for g in grads], opt["lr"])

    for i in range(max(1, min(args.warmup, 1))):
        one_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one_step(i + 1)
    dt = (time.perf_counter() - t0) / args.steps
    value = cores * per_shard / dt
    _, cfg = build_workload(name, 0, config_only=True)
    cfg.update({"workload": name, "parallelism": f"dp{args.gpus}",
                "optimizer": opt.get("kind") if opt else None})
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit,
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
        n, unit, sample = 128, "tokens/s", "1 sequence of 128 tokens, full model widths"
    elif name == "charmlp":
        w = configs.char_mlp(batch=1024, seed=4)
        n, unit, sample = 1024, "samples/s", "batch 1024 of the same graph, 1 step"
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


def tolerance(name, w, plan, feeds):
    """Measured error of the timed config against the oracle, outside the
    timed region: one more step of the same plan runs on the device from the
    network's initial parameters (a fresh parameter set, so the timed run's
    state is left as it is), and the oracle computes the same loss and
    gradients on every host core.  Reported per output as
    max |dev - oracle| / max |oracle|."""
    import oracle
    from poorgrad_b200 import backend
    if name not in ("charmlp", "mlp"):
        return None
    oracle.build()
    oracle.set_threads(os.cpu_count() or 1)
    params = w.network.parameters()
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, feeds, sync=True)
    dev = {g.index: plan.of(g) for g in [w.loss] + list(w.grads)}
    t0 = time.perf_counter()
    ref = oracle.run(w.columns, params, feeds, read=list(dev))
    oracle_s = time.perf_counter() - t0
    oracle.set_threads(1)
    loss_rel = float(abs(dev[w.loss.index] - ref[w.loss.index]) / abs(ref[w.loss.index]))
    grad_rel = max(float(np.abs(dev[g.index] - ref[g.index]).max() /
                         (np.abs(ref[g.index]).max() + 1e-30)) for g in w.grads)
    return {"loss_rel": loss_rel, "grads_max_rel_to_scale": grad_rel,
            "bar": "loss and every gradient within rtol 1e-3 + atol 1e-4 of its scale "
                   "(tests/test_full_size_parity.py)",
            "sample": f"one full-size step ({w.samples} samples) from the initial parameters; "
                      f"oracle {oracle_s:.1f} s on {os.cpu_count()} threads"}


def cublas_baseline(m, k, n, reps=5):
    """The reference's cuda arm for C3 (backend/cuda/kernels/gemm.rs:54-163,
    context.rs:217-288): a fresh cuBLAS handle in its default math mode (no
    TF32), `cublasSgemm_v2` on row-major operands through the column-major
    swap, for C = A.B, dA = dC.B^T and dB = A^T.dC.  Timed device-only (CUDA
    events around the three calls, operands resident) and with the reference's
    per-product copies (pageable host -> device for both operands, the call,
    device -> host of the product, device synchronize; wall clock).  A
    baseline only: nothing of the product path calls cuBLAS."""
    import torch
    lib = None
    for cand in ("libcublas.so.12", "libcublas.so"):
        try:
            lib = C.CDLL(cand)
            break
        except OSError:
            continue
    if lib is None:
        return {"unavailable": "libcublas not found"}
    handle = C.c_void_p()
    if lib.cublasCreate_v2(C.byref(handle)) != 0:
        return {"unavailable": "cublasCreate failed"}
    N, T = 0, 1
    one, zero = C.c_float(1.0), C.c_float(0.0)
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    dC = rng.standard_normal((m, n)).astype(np.float32)

    def sgemm(opb, opa, nn, mm, kk, b, ldb, a, lda, c, ldc):
        rc = lib.cublasSgemm_v2(handle, opb, opa, nn, mm, kk, C.byref(one), C.c_void_p(b), ldb,
                                C.c_void_p(a), lda, C.byref(zero), C.c_void_p(c), ldc)
        assert rc == 0, rc

    # row-major products through the column-major swap: C^T = op(B)^T op(A)^T
    products = [  # (left host, right host, out shape, call)
        (A, B, (m, n), lambda l, r, o: sgemm(N, N, n, m, k, r, n, l, k, o, n)),
        (dC, B, (m, k), lambda l, r, o: sgemm(T, N, k, m, n, r, n, l, n, o, k)),
        (A, dC, (k, n), lambda l, r, o: sgemm(N, T, n, k, m, r, n, l, k, o, n)),
    ]
    dev = [(torch.from_numpy(l).cuda(), torch.from_numpy(r).cuda(),
            torch.empty(shape, device="cuda")) for l, r, shape, _ in products]
    torch.cuda.synchronize()
    flops = 3 * 2.0 * m * n * k

    def device_only():
        for (l, r, o), (_, _, _, call) in zip(dev, products):
            call(l.data_ptr(), r.data_ptr(), o.data_ptr())

    for _ in range(2):
        device_only()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(torch.cuda.default_stream())
    for _ in range(reps):
        device_only()
    e.record(torch.cuda.default_stream())
    torch.cuda.synchronize()
    ms_dev = s.elapsed_time(e) / reps

    def with_copies():
        for (l, r, o), (lh, rh, shape, call) in zip(dev, products):
            l.copy_(torch.from_numpy(lh))
            r.copy_(torch.from_numpy(rh))
            call(l.data_ptr(), r.data_ptr(), o.data_ptr())
            out = o.cpu()
            torch.cuda.synchronize()
        return out

    with_copies()
    t0 = time.perf_counter()
    for _ in range(reps):
        with_copies()
    ms_copy = (time.perf_counter() - t0) * 1e3 / reps
    lib.cublasDestroy_v2(handle)
    return {"device_only": {"ms_per_step": ms_dev, "tflops": flops / ms_dev / 1e9},
            "with_copies": {"ms_per_step": ms_copy, "tflops": flops / ms_copy / 1e9,
                            "copies": "pageable H2D of both operands and D2H of the product, "
                                      "per product"},
            "math_mode": "cuBLAS default (f32, no TF32)", "reps": reps}


def face_with_copies(m, k, n, reps=5):
    """This library's per-task face `tb_gemm_f32` (host slices in, owned
    product out) timed through the same three products as `cublas_baseline`'s
    copy arm (wall clock)."""
    from poorgrad_b200 import backend
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    dC = rng.standard_normal((m, n)).astype(np.float32)

    def step():
        backend.gemm_f32(A, B)
        backend.gemm_f32(dC, B.T)
        backend.gemm_f32(A.T, dC)

    step()
    t0 = time.perf_counter()
    for _ in range(reps):
        step()
    ms = (time.perf_counter() - t0) * 1e3 / reps
    return {"ms_per_step": ms, "tflops": 3 * 2.0 * m * n * k / ms / 1e9,
            "copies": "pageable H2D of both operands and D2H of the product, per product"}


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


# DRAM read + write bytes per launch of the dominant kernel class from one ncu
# capture of the workload (dram__bytes_read.sum + dram__bytes_write.sum), with
# the profile summary it comes from.
NCU_TRAFFIC = {"charmlp": {"gemm": (75.32e6, "profiles/gemm_tcgen05_charmlp_16384x512x512.md: "
                                    "the step's first product, one launch")}}


def traffic(workload, kind):
    return NCU_TRAFFIC.get(workload, {}).get(kind, (None, None))


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
                "frac": achieved / peak, "traffic": traffic(workload, kind)[0],
                "traffic_unit": "bytes per launch", "traffic_source": traffic(workload, kind)[1],
                "timing": "per-kernel CUDA-event replay of the step's kernels, hot cache "
                          "(tbx_profile_kernels)", "launches": len(group),
                "kernel": "k_gemm_tcgen05 (3xTF32, all GEMMs of the step)",
                "share": t * 1e3 / total,
                "peak_note": f"3xTF32-effective = {how} bf16 {bf16:.0f} TF/s / 6"}
    bytes_ = sum(r["read"] + r["write"] for r in group)
    achieved = bytes_ / t / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "traffic": traffic(workload, kind)[0],
            "traffic_unit": "bytes per launch", "traffic_source": traffic(workload, kind)[1],
            "timing": "per-kernel CUDA-event replay of the step's kernels, hot cache "
                      "(tbx_profile_kernels)", "launches": len(group),
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
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch override (profiling)")
    ap.add_argument("--seq", type=int, default=0, help="gpt2 sequence override (profiling)")
    ap.add_argument("--layers", type=int, default=0, help="gpt2 layer override (profiling)")
    ap.add_argument("--bucket-mb", type=float, default=0.0,
                    help="gradient all-reduce bucket size (MiB) for N > 1; 0 = half the "
                         "gradient, between 1 and 32")
    ap.add_argument("--replay-s", type=float, default=1.5,
                    help="untimed replay before the timed steps (clock sampling)")
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

    w, cfg = build_workload(args.config, rank, overrides={
        "batch": args.batch, "seq": args.seq, "layers": args.layers})
    params = w.network.parameters()
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params)
    opt_cfg = w.optimizer
    opt = None
    if opt_cfg:
        opt_kind = {"sgd": backend.SGD, "adam": backend.ADAM, "adamw": backend.ADAMW}[opt_cfg["kind"]]
        opt = backend.Optimizer(plan, dp, opt_kind, zip(w.params, w.grads), opt_cfg["lr"],
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
        # buckets of half the gradient, between 1 and 32 MiB: the small C4
        # gradient (2.2 MB) then goes out in pieces as its writers finish
        # (measured on 2 GPUs: 15 us exposed against 27 us for one bucket)
        if args.bucket_mb <= 0:
            grad_mib = sum(int(np.prod(w.columns.nodes[g.index].shape)) * 4
                           for g in w.grads) / (1 << 20)
            args.bucket_mb = min(32.0, max(1.0, grad_mib / 2))
        comm.attach(plan, bucket_bytes=int(args.bucket_mb * (1 << 20)))

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

    loss_pinned = [torch.zeros((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ready = [torch.cuda.Event() for _ in range(2)]

    def timed(host, clocks=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        plan.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        loss_host = np.empty((), np.float32)
        if clocks:
            clocks.mark("timed_start")
        t_wall = time.perf_counter()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(args.steps):
                step(i, host)
                if host:
                    # D2H of this step's loss into page-locked memory, enqueued
                    # behind the step; the host takes the previous step's loss
                    # while this one runs (every step's loss is read back)
                    slot = i % 2
                    plan.read_async(w.loss, loss_pinned[slot].data_ptr(), 1)
                    loss_ready[slot].record(stream)
                    if i > 0:
                        loss_ready[1 - slot].synchronize()
                        loss_host = loss_pinned[1 - slot].numpy().copy()
            end.record(stream)
            if host and args.steps > 0:
                loss_ready[(args.steps - 1) % 2].synchronize()
                loss_host = loss_pinned[(args.steps - 1) % 2].numpy().copy()
        plan.synchronize()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t_wall) * 1e3
        if clocks:
            clocks.mark("timed_end")
        ms = start.elapsed_time(end)
        t = torch.tensor([ms], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(t.item()), wall, loss_host

    with Clocks(local) as clocks:
        # untimed replay of the same step for >= 1.5 s right before the timed
        # region, so that the clock samples (and any external sampler) see the
        # GPU under this load
        t_end = time.perf_counter() + args.replay_s
        i = 0
        while time.perf_counter() < t_end:
            for _ in range(32):
                step(i)
                i += 1
            plan.synchronize()
        ms, wall, _ = timed(False, clocks)
    ms_e2e, wall_e2e, last_loss = timed(True)
    per_step = ms / args.steps
    metric, unit = metric_of(args.config)
    per_sample = (args.seq or 1024) if args.config == "gpt2" else 1   # tokens per GPT-2 sequence
    samples = w.samples * per_sample * world
    value = samples / (per_step * 1e-3)
    e2e_value = samples / (ms_e2e / args.steps * 1e-3)

    comm_info = None
    if world > 1:
        # exposed exchange time: the same step without the gradient all-reduce
        # (a second plan over the same parameters, no communicator attached),
        # timed the same way; the difference is what the exchange adds
        solo = backend.DevicePlan(w.columns)
        solo_opt = None
        if opt_cfg:
            solo_opt = backend.Optimizer(solo, dp, opt_kind, zip(w.params, w.grads), opt_cfg["lr"],
                                         opt_cfg.get("beta1", 0.9), opt_cfg.get("beta2", 0.999),
                                         opt_cfg.get("eps", 1e-8), opt_cfg.get("decay", 0.0),
                                         gradient_scale=1.0 / world)
        for i in range(3):
            solo.forward(dp, sym_of[i % nb][0])
        solo.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        solo_stream = torch.cuda.ExternalStream(solo.stream())
        s0.record(solo_stream)
        for i in range(args.steps):
            solo.forward(dp, sym_of[i % nb][0])
        s1.record(solo_stream)
        solo.synchronize()
        torch.cuda.synchronize()
        t_solo = torch.tensor([s0.elapsed_time(s1) / args.steps], device="cuda")
        dist.all_reduce(t_solo, op=dist.ReduceOp.MAX)
        grad_bytes = sum(int(np.prod(w.columns.nodes[g.index].shape)) * 4 for g in w.grads)
        comm_info = {"allreduce_bytes_per_step": grad_bytes, "bucket_mib": args.bucket_mb,
                     "step_ms_without_exchange": float(t_solo.item()),
                     "exposed_exchange_ms": per_step - float(t_solo.item()),
                     "how": "the same step on the same rank without the NCCL all-reduce, "
                            "max over ranks; exposed = with - without"}
        del solo_opt, solo
    stats = plan.stats()
    rows = kernel_profile(plan) if rank == 0 and not args.no_kernel_profile else []
    roof = roofline(rows, args.config) if rows else None
    if rank == 0:
        cpu = None if args.no_cpu else cpu_baseline(args.config)
        tol = None if args.no_cpu else tolerance(args.config, w, plan, host_batches[0])
        arena_mb = stats["arena_bytes"] / 2**20
        cfg.update({"workload": args.config, "parallelism": f"dp{world}",
                    "l2": (f"working set > L2: arena {arena_mb:.0f} MiB per step, no flush"
                           if arena_mb > 126 else
                           f"working set {arena_mb:.0f} MiB fits in L2 and is not flushed "
                           "(a small, latency-bound step)"),
                    "optimizer": opt_cfg.get("kind") if opt_cfg else None})
        line = {"metric": metric, "value": value, "unit": unit,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded splitmix64 streams)",
                "config": cfg,
                "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": 4, "wall_ms": wall_e2e,
                        "how": "each step: tb_plan_run with the step's inputs in page-locked "
                               "host memory (copied in on the plan's stream), then its loss "
                               "read back with tb_plan_read_async; the host waits for step i's "
                               "loss after launching step i + 1"},
                "gpu_launches": stats["kernels"] * args.steps,
                "roofline": roof, "cpu_baseline": cpu, "clocks": clocks.summary(),
                "tolerance": tol, "exchange": comm_info,
                "loss": float(last_loss), "wall_ms_timed": wall,
                "kernels_per_step": stats["kernels"], "gemms_per_step": stats["gemms"]}
        if args.config in ("gemm", "gemm_skinny") and not args.no_cpu:
            shape = (4096, 4096, 4096) if args.config == "gemm" else (32768, 768, 3072)
            line["cublas_baseline"] = cublas_baseline(*shape)
            line["face_with_copies"] = face_with_copies(*shape)
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
