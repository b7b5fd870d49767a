#!/usr/bin/env python
"""Benchmark of the fused GLM gradient on B200 (one process per GPU).

Workload (default): one full gradient evaluation of the memory-bound
single-task GLM -- nobs = 2^24 observations, nfeatures = 128, ntargets = 1,
ntasks = 1, float32, X ~ U(-1, 1), beta ~ N(0, 1), y = X beta + N(0, 0.1^2),
lambda2 = 0.01 (lambda = 0.01, alpha = 0).  X is 8 GiB, far larger than L2
(126 MB), so no flush is needed between steps.  Observations are split
into contiguous blocks, one per rank (strong scaling: the total is fixed);
each rank computes its partial sum, the partials are summed with one NCCL
all-reduce, and every rank applies 2*sum + the elastic-net term.

Usage:
    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
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

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "GLM gradient obs·features/s"
UNIT = "obs·features/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--nobs", type=int, default=1 << 24)
    p.add_argument("--nfeatures", type=int, default=128)
    p.add_argument("--lam", type=float, default=0.01)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def workload_config(args, n_gpus):
    return {
        "workload": f"glm_gradient f32 nobs={args.nobs} nfeatures={args.nfeatures} ntargets=1 ntasks=1",
        "nobs": args.nobs,
        "nfeatures": args.nfeatures,
        "ntargets": 1,
        "ntasks": 1,
        "lambda": args.lam,
        "alpha": 0.0,
        "inputs": "X~U(-1,1), beta~N(0,1), y=X beta+N(0,0.1^2), seeded",
        "l2": "inputs larger than L2 (X 8 GiB), no flush",
        "parallelism": f"obs-sharded x{n_gpus} + NCCL all-reduce of the partial gradient" if n_gpus > 1 else "single GPU",
    }


def algorithmic_bytes(nobs, nf, nt=1, ntasks=1, esize=4):
    """X once, Y once, M in and grad out."""
    return esize * (nobs * ntasks * nf + nobs * ntasks * nt + 2 * nf * nt * ntasks)


def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def dram_traffic_per_row():
    """DRAM bytes per observation row of the rows kernel from the committed
    ncu summary (profiles/glm_rows_f32_nf128_traffic.txt), or None."""
    path = os.path.join(REPO, "profiles", "glm_rows_f32_nf128_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_row:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


# --------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm on the host cores
# --------------------------------------------------------------------------
def cpu_sample_rate(nf, rows, lam, reps=3, threads=0):
    """obs·features/s of the oracle's gradient (the reference's host
    algorithm) on `rows` observations; best of `reps`."""
    import numpy as np

    from oracle import pyoracle

    pyoracle.build()
    if threads:
        pyoracle.set_threads(threads)
    rng = np.random.default_rng(7)
    X = rng.uniform(-1, 1, (rows, 1, nf)).astype(np.float32)
    b = rng.normal(size=(1, 1, nf)).astype(np.float32)
    Y = (X[:, 0, :] @ b[0, 0] + rng.normal(0, 0.1, rows)).astype(np.float32).reshape(rows, 1, 1)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        pyoracle.gradient(X, b, Y, lam, 0.0, True)
        best = min(best, time.perf_counter() - t0)
    return rows * nf / best, pyoracle.get_threads(), best


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import pyoracle

    pyoracle.build()
    import numpy as np

    nf = args.nfeatures
    # size each step's sample so the whole run stays near a minute of CPU time
    probe_rows = min(args.nobs, 1 << 21)
    rng = np.random.default_rng(7)
    X = rng.uniform(-1, 1, (probe_rows, 1, nf)).astype(np.float32)
    b = rng.normal(size=(1, 1, nf)).astype(np.float32)
    Y = (X[:, 0, :] @ b[0, 0] + rng.normal(0, 0.1, probe_rows)).astype(np.float32).reshape(probe_rows, 1, 1)
    pyoracle.gradient(X, b, Y, args.lam, 0.0, True)
    t0 = time.perf_counter()
    pyoracle.gradient(X, b, Y, args.lam, 0.0, True)
    t1 = time.perf_counter() - t0
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(probe_rows * min(1.0, budget / max(t1, 1e-9)))
    rows = max(1 << 12, min(probe_rows, rows))
    X, Y = X[:rows], Y[:rows]
    for _ in range(args.warmup):
        pyoracle.gradient(X, b, Y, args.lam, 0.0, True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pyoracle.gradient(X, b, Y, args.lam, 0.0, True)
    dt = time.perf_counter() - t0
    value = rows * nf * args.steps / dt
    sample = f"{rows} of {args.nobs} observations per step (nfeatures={nf}), float32"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(args, args.gpus),
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
        busy = [p for p in window if (num(p[2]) or 0) >= 50] or window
        if not busy:
            busy = [p for (_, p) in self.samples]
        if not busy:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in busy for i in range(4) if p[5 + i].lower().startswith("active")})
        sm = [num(p[0]) for p in busy if num(p[0]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(busy[0][1]), "reasons": reasons, "samples": len(busy),
                "power_w_max": max((num(p[3]) or 0) for p in busy)}


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def make_shard(args, rank, world, device):
    """This rank's rows of the global synthetic problem; blocks of 2^16 rows
    are seeded by their global index, so the data do not depend on N."""
    import torch

    nobs, nf = args.nobs, args.nfeatures
    blk = 1 << 16
    assert nobs % (world * blk) == 0, "nobs must split into 2^16-row blocks per rank"
    per = nobs // world
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    beta = torch.randn((1, 1, nf), generator=g, device=device, dtype=torch.float32)
    X = torch.empty((per, 1, nf), device=device, dtype=torch.float32)
    Y = torch.empty((per, 1, 1), device=device, dtype=torch.float32)
    for i in range(per // blk):
        gb = rank * (per // blk) + i
        g.manual_seed(args.seed * 1_000_003 + gb)
        xs = X[i * blk:(i + 1) * blk]
        xs.uniform_(-1.0, 1.0, generator=g)
        noise = torch.randn((blk,), generator=g, device=device, dtype=torch.float32) * 0.1
        Y[i * blk:(i + 1) * blk, 0, 0] = xs[:, 0, :] @ beta[0, 0] + noise
    return X, Y, beta


def run_ours(args):
    import torch
    import torch.distributed as dist

    from gpu_algos_b200 import capi, glm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    n_gpus = world

    X, Y, beta = make_shard(args, rank, world, device)
    nobs_local, _, nf = X.shape
    ws = torch.empty(glm.workspace_bytes(torch.float32, nf, 1, 1, nobs_local) + 256, dtype=torch.uint8, device=device)
    grad = torch.empty((1, 1, nf), dtype=torch.float32, device=device)
    partial = torch.empty((1, 1, nf), dtype=torch.float64, device=device)
    stream = torch.cuda.current_stream()
    lam = args.lam

    from gpu_algos_b200.sharded import CudaBackend, ShardedGLM

    backend = CudaBackend(workspace=ws)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        if world == 1:
            glm.gradient(X, beta, Y, lam, 0.0, True, out=grad, workspace=ws)
            if ev is not None:
                ev[1].record(stream)
        else:
            backend.partial(X, beta, Y, out=partial)
            if ev is not None:
                ev[1].record(stream)
            dist.all_reduce(partial, op=dist.ReduceOp.SUM)
            backend.finalize(partial, beta, lam, 0.0, grad)

    props = torch.cuda.get_device_properties(device)
    sampler = ClockSampler(f"GPU-{props.uuid}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    kernel_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                     for _ in range(args.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    launches0 = capi.launch_count()
    t_wall0 = time.time()
    start.record(stream)
    for k in range(args.steps):
        step(kernel_events[k])
    end.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    launches = capi.launch_count() - launches0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms_total = start.elapsed_time(end)
    kernel_ms = statistics.mean(a.elapsed_time(b) for (a, b) in kernel_events)
    t = torch.tensor([ms_total, kernel_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, kernel_ms = float(t[0]), float(t[1])
    ms_per_step = ms_total / args.steps
    value = args.nobs * nf / (ms_per_step * 1e-3)

    # end to end through the public API from pinned host buffers
    e2e = None
    if not args.no_e2e:
        Xh = torch.empty(X.shape, dtype=X.dtype, pin_memory=True)
        Yh = torch.empty(Y.shape, dtype=Y.dtype, pin_memory=True)
        Xh.copy_(X)
        Yh.copy_(Y)
        gh = torch.empty(grad.shape, dtype=grad.dtype, pin_memory=True)
        Xd = torch.empty_like(X)
        Yd = torch.empty_like(Y)

        def e2e_step():
            Xd.copy_(Xh, non_blocking=True)
            Yd.copy_(Yh, non_blocking=True)
            if world == 1:
                glm.gradient(Xd, beta, Yd, lam, 0.0, True, out=grad, workspace=ws)
            else:
                ShardedGLM(Xd, Yd, backend).gradient(beta, lam, 0.0, out=grad)
            gh.copy_(grad, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s0.elapsed_time(s1)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te[0]) / args.e2e_steps
        e2e = {"value": args.nobs * nf / (e2e_ms * 1e-3), "unit": UNIT,
               "h2d_bytes_per_step": int(Xh.numel() * 4 + Yh.numel() * 4),
               "d2h_bytes_per_step": int(gh.numel() * 4), "ms_per_step": e2e_ms,
               "steps": args.e2e_steps,
               "path": "pinned host X,Y -> device (cudaMemcpyAsync) -> glmb_gradient_f32 -> host grad"}
        del Xh, Yh, Xd, Yd

    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)

    if world > 1:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = measured_hbm_peak()
        bytes_launch = algorithmic_bytes(nobs_local, nf)
        achieved = bytes_launch / (kernel_ms * 1e-3) / 1e9
        tpr = dram_traffic_per_row()
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                    if peak_kind == "measured" else "fallback 6650 GB/s",
                    "traffic": (tpr * nobs_local) if tpr is not None else None,
                    "algorithmic_bytes": bytes_launch, "kernel_ms": kernel_ms,
                    "kernel": "glm_rows_kernel<float,4,1,1> + glm_finalize_kernel (one glmb_gradient_f32 call)"}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n_gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": workload_config(args, n_gpus), "roofline": roofline,
                "gpu_launches": int(launches), "clocks": clocks}
        if e2e is not None:
            line["e2e"] = e2e
        if n_gpus == 1 and not args.no_cpu_baseline:
            rows = min(args.nobs, 1 << 21)
            rate, cores, secs = cpu_sample_rate(nf, rows, args.lam)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                    "sample": f"{rows} observations x {nf} features float32, best of 3 "
                                              f"({secs * 1e3:.1f} ms each)"}
        print(json.dumps(line), flush=True)
    if world > 1:
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
