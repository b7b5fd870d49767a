#!/usr/bin/env python
"""Benchmark of the GLM path on B200 (one process per GPU).

Default workload ("gradient"): one full gradient evaluation of the
memory-bound single-task GLM -- nobs = 2^24 observations, nfeatures = 128,
ntargets = 1, ntasks = 1, float32, X ~ U(-1, 1), beta ~ N(0, 1),
y = X beta + N(0, 0.1^2), lambda2 = 0.01 (lambda = 0.01, alpha = 0).  X is
8 GiB, far larger than L2 (126 MB), so no flush is needed between steps.
Observations are split into contiguous blocks, one per rank (strong scaling:
the total is fixed); each rank computes its partial sum, the partials are
summed with one NCCL all-reduce, and every rank applies 2*sum + the
elastic-net term.

Other workloads (--workload):
  driver     nobs 8192, nfeatures 32, float32: the reference driver's
             CPU-checkable shape (too small to shard: replicas per GPU)
  multitask  64 tasks x 2^18 observations x 256 features x 16 targets,
             float64 (tasks sharded across ranks, no collective)
  gradient_f16  the default workload with float16 X, y and model (float
             arithmetic in the kernel; half the HBM bytes per row)
  gradient_bf16 the same with bfloat16
  dense      wide dense gradient on the tensor cores (3xTF32): nobs 2^20,
             nfeatures 4096, ntargets 256, float32, X ~ U(-1,1)/sqrt(4096),
             lambda2 0.001 (observations sharded)
  fit        elastic-net fit, 20 power iterations + 200 ISTA steps,
             nobs 2^26, nfeatures 512, float32, lambda1 0.05, lambda2 0.01,
             10 %-sparse true coefficients (observations sharded)

Usage:
    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line.  `--impl reference` times the reference's CPU
algorithm (the oracle port: the reference's C++ host path cannot be built
here) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "GLM gradient obs·features/s"
UNIT = "obs·features/s"
FALLBACK_HBM_GBS = 6650.0
HOST_PIN_LIMIT = 40 << 30  # largest per-rank X copied through pinned host memory for e2e


@dataclass(frozen=True)
class Workload:
    name: str
    nobs: int
    nf: int
    nt: int
    ntasks: int
    dtype: str  # "f16" | "bf16" | "f32" | "f64"
    x: str  # "uniform" (U(-1,1)) | "normal" (N(0,1)), times x_scale
    noise: float
    shard: str  # "obs" | "tasks" | "replica"
    kind: str = "gradient"  # "gradient" | "fit"
    lam: float = 0.0
    alpha: float = 0.0
    independent_beta: bool = False  # gradient at a model other than the true one
    sparsity: float = 1.0  # fraction of non-zero true coefficients
    lambda1: float = 0.0
    lambda2: float = 0.0
    n_power: int = 0
    n_iter: int = 0
    block: int = 1 << 16  # rows per seeded generation block
    x_scale: float = 1.0


WORKLOADS = {
    "gradient": Workload("gradient", 1 << 24, 128, 1, 1, "f32", "uniform", 0.1, "obs", lam=0.01),
    "driver": Workload("driver", 8192, 32, 1, 1, "f32", "uniform", 0.01, "replica", lam=0.1,
                       independent_beta=True, block=8192),
    "multitask": Workload("multitask", 1 << 18, 256, 16, 64, "f64", "normal", 0.05, "tasks", lam=0.1,
                          independent_beta=True, block=1 << 14),
    "gradient_f16": Workload("gradient_f16", 1 << 24, 128, 1, 1, "f16", "uniform", 0.1, "obs", lam=0.01),
    "gradient_bf16": Workload("gradient_bf16", 1 << 24, 128, 1, 1, "bf16", "uniform", 0.1, "obs", lam=0.01),
    "dense": Workload("dense", 1 << 20, 4096, 256, 1, "f32", "uniform", 0.01, "obs", lam=0.001,
                      x_scale=4096 ** -0.5, block=1 << 15),
    "fit": Workload("fit", 1 << 26, 512, 1, 1, "f32", "normal", 0.1, "obs", kind="fit", sparsity=0.1,
                    lambda1=0.05, lambda2=0.01, n_power=20, n_iter=200),
}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default: per workload)")
    p.add_argument("--warmup", type=int, default=None)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="gradient")
    p.add_argument("--nobs", type=int, default=None, help="override the workload's nobs")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-graph", action="store_true",
                   help="launch every step from the host instead of replaying a captured CUDA graph")
    p.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                   help="cross-GPU sum of the partial gradient: library peer-memory exchange or NCCL all-reduce")
    a = p.parse_args()
    w = WORKLOADS[a.workload]
    if a.nobs is not None:
        w = Workload(**{**w.__dict__, "nobs": a.nobs, "block": min(w.block, a.nobs)})
    a.w = w
    default_steps = {"gradient": 500, "gradient_f16": 500, "gradient_bf16": 500, "driver": 2000, "multitask": 20,
                     "dense": 20, "fit": 2}[w.name]
    a.steps = a.steps if a.steps is not None else default_steps
    a.warmup = a.warmup if a.warmup is not None else (1 if w.kind == "fit" else 10)
    return a


def passes_per_step(w: Workload) -> int:
    return (w.n_power + w.n_iter) if w.kind == "fit" else 1


def workload_config(w: Workload, n_gpus: int, exchange: str = "peer") -> dict:
    cfg = {
        "workload": (f"glm_{'fit_elastic_net' if w.kind == 'fit' else 'gradient'} {w.dtype} nobs={w.nobs} "
                     f"nfeatures={w.nf} ntargets={w.nt} ntasks={w.ntasks}"),
        "nobs": w.nobs, "nfeatures": w.nf, "ntargets": w.nt, "ntasks": w.ntasks,
        "inputs": (f"X~{'U(-1,1)' if w.x == 'uniform' else 'N(0,1)'}"
                   + (f"/sqrt({w.nf})" if w.x_scale != 1.0 else "") + ", beta~N(0,1)"
                   + (f" {int(w.sparsity * 100)}%-sparse" if w.sparsity < 1 else "")
                   + f", y=X beta+N(0,{w.noise}^2), seeded"),
        "l2": "inputs larger than L2 (126 MB), no flush" if w.nobs * w.ntasks * w.nf * 4 > (256 << 20)
              else "inputs smaller than L2 (launch-bound shape)",
    }
    if w.kind == "fit":
        cfg.update(lambda1=w.lambda1, lambda2=w.lambda2, n_power=w.n_power, n_iter=w.n_iter)
    else:
        cfg.update({"lambda": w.lam, "alpha": w.alpha})
    if n_gpus == 1:
        cfg["parallelism"] = "single GPU"
    elif w.shard == "obs":
        cfg["parallelism"] = (f"obs-sharded x{n_gpus} + one NCCL all-reduce of the partial gradient per pass"
                              if exchange == "nccl" else
                              f"obs-sharded x{n_gpus}; partials summed over NVLink peer memory by the "
                              "library's exchange kernel (P2P stores + flags), one per pass")
    elif w.shard == "tasks":
        cfg["parallelism"] = f"tasks-sharded x{n_gpus}, no collective"
    else:
        cfg["parallelism"] = f"{n_gpus} independent replicas (shape too small to shard)"
    return cfg


def algorithmic_bytes(nobs, nf, nt, ntasks, esize):
    """X once, Y once, M in and grad out."""
    return esize * (nobs * ntasks * nf + nobs * ntasks * nt + 2 * nf * nt * ntasks)


def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_bf16_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return None


def dram_traffic_per_row(w: Workload):
    """DRAM bytes per observation row of the measured call, from the
    committed ncu summary of that kernel and shape, or None."""
    name = {"gradient": "glm_rows_f32_nf128_traffic.txt",
            "dense": "glm_dense_f32_nf4096_nt256_traffic.txt"}.get(w.name)
    if name is None:
        return None
    try:
        with open(os.path.join(REPO, "profiles", name)) as f:
            for line in f:
                if line.startswith(("dram_bytes_per_row:", "dram_bytes_per_obs:")):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# --------------------------------------------------------------------------
# CPU: the reference's algorithm (oracle port) on the host cores
# --------------------------------------------------------------------------
def cpu_problem(w: Workload, rows: int):
    """Host copy of a `rows`-observation sample (bfloat16 as uint16 bit patterns)."""
    import numpy as np

    rng = np.random.default_rng(7)
    if w.dtype == "bf16":
        from oracle import pyoracle

        dt, conv, back = np.float32, pyoracle.bf16_bits, pyoracle.bf16_to_f32
    else:
        dt = {"f16": np.float16, "f32": np.float32, "f64": np.float64}[w.dtype]
        conv = back = (lambda a: a)  # noqa: E731
    if w.x == "uniform":
        X = rng.uniform(-1, 1, (rows, w.ntasks, w.nf)).astype(dt)
    else:
        X = rng.normal(size=(rows, w.ntasks, w.nf)).astype(dt)
    X = conv(X * dt(w.x_scale))
    b = conv(rng.normal(size=(w.ntasks, w.nt, w.nf)).astype(dt))
    Y = conv((np.einsum("otf,tkf->otk", back(X).astype(np.float64), back(b).astype(np.float64))
              + w.noise * rng.normal(size=(rows, w.ntasks, w.nt))).astype(dt))
    return X, b, Y


def cpu_pass(pyoracle, w: Workload, X, b, Y):
    bf16 = w.dtype == "bf16"
    if w.kind == "fit":
        return pyoracle.gradient(X, b, Y, w.lambda2, 0.0, True, bf16=bf16)
    return pyoracle.gradient(X, b, Y, w.lam, w.alpha, True, bf16=bf16)


def cpu_sample_rate(w: Workload, rows: int, reps: int = 3):
    """obs·features/s of one oracle pass (the reference's host algorithm)
    over `rows` observations on all host threads; best of `reps`."""
    from oracle import pyoracle

    pyoracle.build()
    pyoracle.set_threads(host_threads())
    X, b, Y = cpu_problem(w, rows)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        cpu_pass(pyoracle, w, X, b, Y)
        best = min(best, time.perf_counter() - t0)
    return rows * w.ntasks * w.nf / best, pyoracle.get_threads(), best


def cpu_rows(w: Workload) -> int:
    return min(w.nobs, {"gradient": 1 << 21, "gradient_f16": 1 << 20, "gradient_bf16": 1 << 20, "driver": 8192,
                        "multitask": 4096, "dense": 4096, "fit": 1 << 19}[w.name])


def run_reference(args):
    w = args.w
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    from oracle import pyoracle

    pyoracle.build()
    pyoracle.set_threads(host_threads())
    rows = cpu_rows(w)
    X, b, Y = cpu_problem(w, rows)
    cpu_pass(pyoracle, w, X, b, Y)
    t0 = time.perf_counter()
    cpu_pass(pyoracle, w, X, b, Y)
    t1 = time.perf_counter() - t0
    # each step is a bounded sample: keep the whole run near a minute of CPU time
    cpu_seconds = 60.0 / max(1, args.steps + args.warmup)
    rows = max(min(rows, 64), int(rows * min(1.0, cpu_seconds / max(t1, 1e-9))))
    X, Y = X[:rows], Y[:rows]
    for _ in range(args.warmup):
        cpu_pass(pyoracle, w, X, b, Y)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_pass(pyoracle, w, X, b, Y)
    dt = time.perf_counter() - t0
    value = rows * w.ntasks * w.nf * args.steps / dt
    sample = (f"{rows} of {w.nobs} observations x {w.ntasks} tasks x {w.nf} features per step, {w.dtype}"
              + (", one gradient pass of the fit" if w.kind == "fit" else ""))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic", "config": workload_config(w, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": pyoracle.get_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,utilization.gpu,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def wait_first(self, timeout_s: float = 5.0):
        """Block until nvidia-smi has delivered a sample (or the timeout)."""
        t_end = time.time() + timeout_s
        while self.proc is not None and not self.samples and time.time() < t_end:
            time.sleep(0.02)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        window = [p for (t, p) in self.samples if t0 <= t <= t1]
        where = "timed region"
        if not window:  # a timed region shorter than the sampling period: the samples next to it
            window = [p for (t, p) in self.samples if t0 - 0.5 <= t <= t1 + 0.5]
            where = "within 0.5 s of the timed region"
        busy = [p for p in window if (num(p[2]) or 0) >= 50] or window
        if not busy:
            busy = [p for (_, p) in self.samples]
            where = "whole run"
        if not busy:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in busy for i in range(4) if p[5 + i].lower().startswith("active")})
        sm = [num(p[0]) for p in busy if num(p[0]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(busy[0][1]), "reasons": reasons, "samples": len(busy), "sampled": where,
                "power_w_max": max((num(p[3]) or 0) for p in busy)}


# --------------------------------------------------------------------------
# synthetic data, generated on the device
# --------------------------------------------------------------------------
def make_local(w: Workload, rank: int, world: int, seed: int, device):
    """This rank's part of the global synthetic problem.  Blocks of rows
    (per task) are seeded by their global index, so the data a rank holds do
    not depend on the number of ranks."""
    import torch

    from gpu_algos_b200.sharded import obs_range, task_range

    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32, "f64": torch.float64}[w.dtype]
    if w.shard == "obs":
        assert w.nobs % (world * w.block) == 0, "nobs must split into whole generation blocks per rank"
        lo, hi = obs_range(w.nobs, world, rank)
        t_lo, t_hi = 0, w.ntasks
    elif w.shard == "tasks":
        lo, hi = 0, w.nobs
        t_lo, t_hi = task_range(w.ntasks, world, rank)
    else:
        lo, hi, t_lo, t_hi = 0, w.nobs, 0, w.ntasks
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    beta_true = torch.randn((w.ntasks, w.nt, w.nf), generator=g, device=device, dtype=torch.float64)
    if w.sparsity < 1:
        keep = torch.rand((w.ntasks, w.nt, w.nf), generator=g, device=device, dtype=torch.float64) < w.sparsity
        beta_true = beta_true * keep
    beta_eval = (torch.randn((w.ntasks, w.nt, w.nf), generator=g, device=device, dtype=torch.float64)
                 if w.independent_beta else beta_true.clone())
    nloc, tloc = hi - lo, t_hi - t_lo
    X = torch.empty((nloc, tloc, w.nf), device=device, dtype=dt)
    Y = torch.empty((nloc, tloc, w.nt), device=device, dtype=dt)
    for j in range(tloc):
        task = t_lo + j
        bt = beta_true[task].to(dt)  # (nt, nf)
        for b0 in range(lo, hi, w.block):
            rows = min(w.block, hi - b0)
            g.manual_seed(seed * 1_000_003 + task * 1_000_000_007 + b0 // w.block)
            xs = torch.empty((rows, w.nf), device=device, dtype=dt)
            if w.x == "uniform":
                xs.uniform_(-1.0, 1.0, generator=g)
            else:
                xs.normal_(generator=g)
            if w.x_scale != 1.0:
                xs *= w.x_scale
            noise = torch.randn((rows, w.nt), generator=g, device=device, dtype=dt) * w.noise
            X[b0 - lo:b0 - lo + rows, j, :] = xs
            Y[b0 - lo:b0 - lo + rows, j, :] = xs @ bt.T + noise
    M = beta_eval[t_lo:t_hi].to(dt).contiguous()
    return X, Y, M, (lo, hi, t_lo, t_hi)


def measured_fp64_tflops(device, sustained_s: float = 0.3):
    """cuBLAS DGEMM throughput measured here (the FP64 roofline denominator;
    MEASURED_PEAKS.json has no FP64 figure): (burst, sustained), as for TF32."""
    import torch

    n = 8192
    a = torch.randn((n, n), device=device, dtype=torch.float64)
    b = torch.randn((n, n), device=device, dtype=torch.float64)
    c = torch.empty((n, n), device=device, dtype=torch.float64)
    torch.matmul(a, b, out=c)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    reps = max(3, int(sustained_s / (best * 1e-3)))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch.matmul(a, b, out=c)
    e1.record()
    torch.cuda.synchronize()
    sustained = 2.0 * n ** 3 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
    del a, b, c
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12, sustained


def measured_tf32_tflops(device, sustained_s: float = 0.5):
    """cuBLAS TF32 GEMM throughput measured here (the tensor-pipe denominator
    of the 3xTF32 path; MEASURED_PEAKS.json has bf16 only): (burst, sustained)
    -- the best of 5 single GEMMs, and back-to-back GEMMs for about
    `sustained_s` seconds, the regime (power cap, clocks) of a kernel timed
    inside a long run."""
    import torch

    n = 8192
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn((n, n), device=device, dtype=torch.float32)
        b = torch.randn((n, n), device=device, dtype=torch.float32)
        c = torch.empty((n, n), device=device, dtype=torch.float32)
        torch.matmul(a, b, out=c)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        reps = max(5, int(sustained_s / (best * 1e-3)))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        sustained = 2.0 * n ** 3 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
        del a, b, c
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12, sustained


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    from gpu_algos_b200 import capi, glm
    from gpu_algos_b200.sharded import CudaBackend, ShardedGLM

    w = args.w
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        # keep stdout for the one JSON line: whatever NCCL_DEBUG asks NCCL to
        # print (its version, INIT lines with the rank count, ...) goes to stderr
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    n_gpus = world
    collective = world > 1 and w.shard == "obs"

    X, Y, M, _ = make_local(w, rank, world, args.seed, device)
    nobs_l, ntasks_l, nf = X.shape
    nt = Y.shape[2]
    dt = X.dtype
    esize = X.element_size()
    ws_bytes = glm.workspace_bytes(dt, nf, nt, ntasks_l, nobs_l)
    if w.kind == "fit":
        ws_bytes = max(ws_bytes, int(getattr(capi.lib(), f"glmb_fit_workspace_size_{glm.SUFFIX[dt]}")(
            nf, nt, ntasks_l, nobs_l)))
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=device)
    grad = torch.empty((ntasks_l, nt, nf), dtype=dt, device=device)
    partial = torch.empty((ntasks_l, nt, nf), dtype=torch.float64, device=device)
    beta_fit = torch.empty((ntasks_l, nt, nf), dtype=dt, device=device)
    lip = torch.empty((ntasks_l,), dtype=torch.float64, device=device)
    stream = torch.cuda.current_stream()
    peer = None
    if collective and args.exchange == "peer":
        from gpu_algos_b200.sharded import PeerBackend, PeerGroup

        peer = PeerGroup(max_elems=ntasks_l * nt * nf, timeout_ms=5000.0)
        backend = PeerBackend(peer, workspace=ws)
    else:
        backend = CudaBackend(workspace=ws)

    def gradient_step(Xs, Ys, ev=None):
        if ev is not None:
            ev[0].record(stream)
        if not collective:
            glm.gradient(Xs, M, Ys, w.lam, w.alpha, True, out=grad, workspace=ws)
            if ev is not None:
                ev[1].record(stream)
        elif peer is not None:
            backend.reduced_gradient(Xs, M, Ys, w.lam, w.alpha, grad, None)
            if ev is not None:
                ev[1].record(stream)
        else:
            backend.partial(Xs, M, Ys, out=partial)
            if ev is not None:
                ev[1].record(stream)
            dist.all_reduce(partial, op=dist.ReduceOp.SUM)
            backend.finalize(partial, M, w.lam, w.alpha, grad)

    def fit_step(Xs, Ys, ev=None):
        if ev is not None:
            ev[0].record(stream)
        if world == 1:
            glm.fit_elastic_net(Xs, Ys, w.lambda1, w.lambda2, w.n_power, w.n_iter, seed=args.seed,
                                beta=beta_fit, lipschitz=lip, workspace=ws)
        else:
            b, L = ShardedGLM(Xs, Ys, backend).fit_elastic_net(w.lambda1, w.lambda2, w.n_power, w.n_iter,
                                                               seed=args.seed)  # peer or NCCL exchange
            beta_fit.copy_(b)
            lip.copy_(L)
        if ev is not None:
            ev[1].record(stream)

    step = fit_step if w.kind == "fit" else gradient_step

    fp64_burst, fp64_peak = measured_fp64_tflops(device) if (w.dtype == "f64" and rank == 0) else (None, None)
    tf32_burst, tf32_peak = measured_tf32_tflops(device) if (w.name == "dense" and rank == 0) else (None, None)
    props = torch.cuda.get_device_properties(device)
    sampler = ClockSampler(f"GPU-{props.uuid}")
    sampler.wait_first()

    for _ in range(args.warmup):
        step(X, Y)
    torch.cuda.synchronize()
    # Gradient workloads on one GPU or with the peer exchange: the K timed
    # steps (2-4 launches each) are captured into one CUDA graph and replayed
    # once, back to back as a fit would issue them, so the per-step cost is the
    # kernels' and not the host's launch overhead.  The exchange keeps its
    # call number in device memory, so every step of the graph is a new
    # exchange.  (NCCL steps are collectives issued by torch.distributed:
    # host-launched, timed per step.)
    graph = None
    host_step = step  # the public call, launched from the host (used by e2e)
    if w.kind == "gradient" and not args.no_graph and (world == 1 or peer is not None or not collective):
        graph = torch.cuda.CUDAGraph()
        c0 = capi.launch_count()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                step(X, Y)
        launches_per_graph = capi.launch_count() - c0
        graph.replay()  # upload; its K steps are further warm-up
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if world > 1:
        # device-side rendezvous: the ranks' start events are recorded once
        # every rank's GPU has reached this all-reduce, so host launch skew
        # after the barrier does not land in the first timed step
        dist.all_reduce(torch.zeros(1, device=device))

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    launches0 = capi.launch_count()
    t_wall0 = time.time()
    if graph is not None:
        start.record(stream)
        graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
    else:
        kernel_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                         for _ in range(args.steps)]
        start.record(stream)
        for k in range(args.steps):
            step(X, Y, kernel_events[k])
        end.record(stream)
        torch.cuda.synchronize()
    t_wall1 = time.time()
    launches = launches_per_graph if graph is not None else capi.launch_count() - launches0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms_total = start.elapsed_time(end)
    if graph is not None:
        kernel_ms = ms_total / args.steps  # the graph holds the gradient calls and nothing else
    else:
        kernel_ms = statistics.mean(a.elapsed_time(b) for (a, b) in kernel_events)
    t = torch.tensor([ms_total, kernel_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, kernel_ms = float(t[0]), float(t[1])
    ms_per_step = ms_total / args.steps
    passes = passes_per_step(w)
    units_per_pass = w.nobs * w.ntasks * w.nf * (world if w.shard == "replica" else 1)
    value = units_per_pass * passes / (ms_per_step * 1e-3)

    # end to end through the public API from pinned host buffers
    e2e = None
    if not args.no_e2e and X.numel() * esize <= HOST_PIN_LIMIT:
        Xh = torch.empty(X.shape, dtype=dt, pin_memory=True)
        Yh = torch.empty(Y.shape, dtype=dt, pin_memory=True)
        Xh.copy_(X)
        Yh.copy_(Y)
        out = beta_fit if w.kind == "fit" else grad
        oh = torch.empty(out.shape, dtype=dt, pin_memory=True)
        Xd = torch.empty_like(X)
        Yd = torch.empty_like(Y)

        def e2e_step():
            Xd.copy_(Xh, non_blocking=True)
            Yd.copy_(Yh, non_blocking=True)
            host_step(Xd, Yd)
            oh.copy_(out, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        n_e2e = max(1, min(args.e2e_steps, args.steps))
        s0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        # the host link's own ceiling for the same bytes: the two copies alone
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        c0.record(stream)
        for _ in range(n_e2e):
            Xd.copy_(Xh, non_blocking=True)
            Yd.copy_(Yh, non_blocking=True)
        c1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s0.elapsed_time(s1), c0.elapsed_time(c1)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te[0]) / n_e2e
        copy_ms = float(te[1]) / n_e2e
        h2d_bytes = int((Xh.numel() + Yh.numel()) * esize)
        e2e = {"value": units_per_pass * passes / (e2e_ms * 1e-3), "unit": UNIT,
               "h2d_bytes_per_step": h2d_bytes,
               "d2h_bytes_per_step": int(oh.numel() * esize), "ms_per_step": e2e_ms, "steps": n_e2e,
               "path": "pinned host X,Y -> device (cudaMemcpyAsync) -> "
                       + ("glmb_fit_elastic_net" if w.kind == "fit" else "glmb_gradient") + " -> host result",
               "h2d_ceiling": {"ms_per_step": copy_ms, "gbs_per_gpu": h2d_bytes / (copy_ms * 1e-3) / 1e9,
                               "value": units_per_pass * passes / (copy_ms * 1e-3),
                               "what": "the same pinned host->device copies alone, max over ranks"},
               "frac_of_h2d_ceiling": copy_ms / e2e_ms}
        del Xh, Yh, Xd, Yd

    # the sharded step's two parts, each as K back-to-back calls in one graph:
    # this rank's pass alone (rows + finalize, no exchange) and the exchange
    # alone (the same sharded call on zero local rows); max over ranks
    breakdown = None
    if peer is not None and graph is not None:
        def graph_ms(fn):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(args.steps):
                    fn()
            g.replay()
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            dist.all_reduce(torch.zeros(1, device=device))
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            torch.cuda.synchronize()
            del g
            return a.elapsed_time(b) / args.steps

        local_ms = graph_ms(lambda: glm.gradient(X, M, Y, w.lam, w.alpha, True, out=grad, workspace=ws))
        X0, Y0 = X[:0], Y[:0]
        exchange_ms = graph_ms(lambda: backend.reduced_gradient(X0, M, Y0, w.lam, w.alpha, grad, None))
        tb = torch.tensor([local_ms, exchange_ms], dtype=torch.float64, device=device)
        dist.all_reduce(tb, op=dist.ReduceOp.MAX)
        breakdown = {"local_pass_us": float(tb[0]) * 1e3, "exchange_only_us": float(tb[1]) * 1e3,
                     "step_us": ms_per_step * 1e3,
                     "what": "per call, K calls in one graph, max over ranks: the rank's own rows pass + "
                             "finalize without exchange; the sharded call on zero local rows (exchange alone)"}

    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)

    if world > 1:
        dist.barrier()
    if rank == 0:
        hbm_peak, peak_kind = measured_hbm_peak()
        bytes_pass = algorithmic_bytes(nobs_l, nf, nt, ntasks_l, esize)
        hbm_achieved = bytes_pass * passes / (kernel_ms * 1e-3) / 1e9
        tpr = dram_traffic_per_row(w)
        peak_note = ("measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s")
        kernel_name = {"gradient": "glm_rows_kernel (+ finalize): one glmb_gradient call",
                       "gradient_f16": "glm_rows_kernel<__half> (+ finalize): one glmb_gradient_f16 call",
                       "gradient_bf16": "glm_rows_kernel<__nv_bfloat16> (+ finalize): one glmb_gradient_bf16 call",
                       "driver": "glm_rows_kernel (+ finalize): one glmb_gradient call",
                       "multitask": "glm_tiles_f64_kernel (+ finalize): one glmb_gradient_f64 call",
                       "dense": "glm_dense_gemm_kernel x2 on CTA pairs (GEMM1 residuals, GEMM2 split-K X^T R) "
                                "+ split reduction: one glmb_gradient call",
                       "fit": f"whole fit: {passes} passes of glm_rows_kernel + finalize/prox kernels"}[w.name]
        if collective and w.kind == "gradient" and w.name != "dense":
            kernel_name = ("glm_rows_kernel + glm_exchange_kernel: one glmb_gradient_sharded call"
                           if peer is not None else
                           "glm_rows_kernel (+ partial reduction): one glmb_gradient_partial call")
        if w.name == "multitask":
            flops = 4.0 * nobs_l * ntasks_l * nf * nt
            achieved = flops / (kernel_ms * 1e-3) / 1e12
            roofline = {"bound": "tensor", "achieved": achieved, "peak": fp64_peak, "unit": "TFLOP/s",
                        "frac": achieved / fp64_peak,
                        "peak_kind": (f"measured here: cuBLAS DGEMM 8192^3 back to back for 0.3 s = {fp64_peak:.1f} "
                                      f"TFLOP/s (burst {fp64_burst:.1f}); MEASURED_PEAKS.json has no FP64 figure"),
                        "frac_of_burst": achieved / fp64_burst,
                        "traffic": None, "algorithmic_flops": flops, "kernel_ms": kernel_ms, "kernel": kernel_name,
                        "hbm_achieved_gbs": hbm_achieved, "hbm_frac": hbm_achieved / hbm_peak}
        elif w.name == "dense":
            # algorithmic fp32 FLOPs (two contractions); the tensor pipe runs 3 tf32 MMAs per product
            flops = 4.0 * nobs_l * ntasks_l * nf * nt
            achieved = flops / (kernel_ms * 1e-3) / 1e12
            peak = tf32_peak / 3.0
            roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak,
                        "peak_kind": (f"measured here: cuBLAS TF32 GEMM 8192^3 back to back for 0.5 s (the regime "
                                      f"of this {args.steps}-step run) = {tf32_peak:.1f} TFLOP/s, / 3 for 3xTF32; "
                                      f"burst (best single GEMM) {tf32_burst:.1f} TFLOP/s; MEASURED_PEAKS.json has "
                                      f"bf16 only ({measured_bf16_peak()} burst)"),
                        "frac_of_burst": achieved / (tf32_burst / 3.0),
                        "tf32_pipe_achieved": 3.0 * achieved, "tf32_peak": tf32_peak, "tf32_peak_burst": tf32_burst,
                        "traffic": (tpr * nobs_l) if tpr is not None else None, "algorithmic_flops": flops, "kernel_ms": kernel_ms, "kernel": kernel_name,
                        "hbm_achieved_gbs": hbm_achieved, "hbm_frac": hbm_achieved / hbm_peak}
        else:
            roofline = {"bound": "hbm", "achieved": hbm_achieved, "peak": hbm_peak, "unit": "GB/s",
                        "frac": hbm_achieved / hbm_peak, "peak_kind": peak_note,
                        "traffic": (tpr * nobs_l) if tpr is not None else None,
                        "algorithmic_bytes": bytes_pass * passes, "kernel_ms": kernel_ms, "kernel": kernel_name}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n_gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if w.shard != "replica" else "weak", "vs_baseline": None,
                "dtype": w.dtype, "data": "synthetic", "config": workload_config(w, n_gpus, args.exchange),
                "roofline": roofline, "gpu_launches": int(launches), "clocks": clocks,
                "step_launch": (f"the {args.steps} timed calls captured in one CUDA graph, replayed once"
                                if graph is not None else "host launches")}
        if w.kind == "fit":
            line["fit"] = {"passes_per_step": passes, "ms_per_pass": ms_per_step / passes,
                           "lipschitz": float(lip[0].item()), "nonzero": int((beta_fit != 0).sum().item())}
        if e2e is not None:
            line["e2e"] = e2e
        if breakdown is not None:
            line["breakdown"] = breakdown
        if n_gpus == 1 and not args.no_cpu_baseline:
            rows = cpu_rows(w)
            rate, cores, secs = cpu_sample_rate(w, rows)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                    "sample": f"{rows} observations x {w.ntasks} tasks x {w.nf} features "
                                              f"{w.dtype}, one pass, best of 3 ({secs * 1e3:.1f} ms each)"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if peer is not None:
            if peer.status() != 0:
                print("[bench] a peer exchange wait ran out", file=sys.stderr)
            peer.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
