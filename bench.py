#!/usr/bin/env python3
"""Benchmark driver (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads:
  q4_gemv   config 0 -- one step = 32 Q4_0 x Q8 GEMVs, one over each of 32
            copies of a 4096x4096 weight (303 MB, 2.4x the 126 MB L2, so every
            launch streams its weight from HBM), metric HBM GB/s.

--clock-window S keeps the same CUDA graph running for S seconds right
before the timed region so nvidia-smi has samples under load (the timed
region itself is unchanged).

Multi-GPU: one process per GPU under torchrun; every rank runs its own
replica of the workload (the GEMV does not shard), timing is the max over
ranks and `value` sums the work of all ranks.

`--impl reference` times the reference's own CPU code (oracle/_ref, built
from the unmodified reference sources) on this host's cores, same metric.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


# ----------------------------------------------------------------- helpers

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]), "power": float(parts[3]),
                             "hw": parts[5], "hwt": parts[6], "swt": parts[7], "pcap": parts[8]})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        load = [r for r in rows if r["power"] > 200] or rows
        reasons = sorted({name for r in load for name, key in
                          (("hw_slowdown", "hw"), ("hw_thermal_slowdown", "hwt"), ("sw_thermal_slowdown", "swt"),
                           ("sw_power_cap", "pcap")) if r[key].lower() == "active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": load[0]["max"],
                "reasons": reasons, "samples": len(load)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def all_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def traffic_from_profiles(kernel_key: str):
    """DRAM bytes per launch recorded from an ncu capture (profiles/traffic.json)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(kernel_key, {}).get("dram_bytes_per_launch")


# -------------------------------------------------------- q4_gemv (config 0)

Q4_ROWS = Q4_COLS = 4096
Q4_W_BYTES = Q4_ROWS * (Q4_COLS // 32) * 18
Q4_ALG_BYTES = Q4_W_BYTES + Q4_COLS * 4 + Q4_ROWS * 4   # weights once + x in + y out
Q4_COPIES = 32                                           # 32 x 9.47 MB = 303 MB, 2.4x the L2


def q4_inputs(seed=1234):
    from memvanta_b200 import gguf
    rng = np.random.default_rng(seed)
    ws = [gguf.gen_q4_0(Q4_ROWS, Q4_COLS, rng) for _ in range(Q4_COPIES)]
    x = rng.standard_normal(Q4_COLS).astype(np.float32)
    return ws, x


def run_q4_gemv_ours(args, world, rank, local):
    import torch
    import memvanta_b200 as mv
    mv.init(local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ws, x = q4_inputs()
    W = [mv.Weight.upload(w, mv.Q4_0, Q4_ROWS, Q4_COLS) for w in ws]
    xd = torch.from_numpy(x).to(dev)
    ys = [torch.empty(Q4_ROWS, dtype=torch.float32, device=dev) for _ in range(Q4_COPIES)]
    stream = torch.cuda.Stream(device=dev)

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            mv.gemv(W[0], xd, ys[0], stream)   # warm the launch path before capture
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    mv.gemv(W[i % Q4_COPIES], xd, ys[i % Q4_COPIES], stream)
        return g

    launches = args.steps * Q4_COPIES
    g_warm, g_timed = capture(args.warmup * Q4_COPIES), capture(launches)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # graphs replay on the current stream: keep it the stream the events use
    with torch.cuda.stream(stream):
        g_warm.replay()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            t_end = time.perf_counter() + args.clock_window
            while time.perf_counter() < t_end:
                g_warm.replay()
                torch.cuda.synchronize()
            barrier(world)
            torch.cuda.synchronize()
            e0.record(stream)
            g_timed.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    ms = all_max(ms, world)
    # correctness spot check of the timed path
    y_ref = ys[0].clone()
    mv.gemv(W[0], xd, y_ref, stream)
    torch.cuda.synchronize()
    assert torch.equal(y_ref, ys[0])
    per_launch_s = ms / 1e3 / launches
    gbs = Q4_ALG_BYTES / per_launch_s / 1e9
    # e2e: the reference-facing host-pointer call (tensor_matvec contract)
    y_host = np.empty(Q4_ROWS, np.float32)
    for _ in range(3):
        y_host = mv.tensor_matvec(W[0], x)
    n_e2e = 200
    barrier(world)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        y_host = mv.tensor_matvec(W[i % Q4_COPIES], x)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    e2e_s = all_max(e2e_s, world)
    return {"ms_total": ms, "per_launch_s": per_launch_s, "gbs": gbs, "e2e_gbs": Q4_ALG_BYTES / e2e_s / 1e9,
            "clocks": clk.summary(), "gpu_launches": launches}


def run_q4_gemv_cpu(seconds=8.0):
    """The reference's tensor_matvec (oracle/_ref) on this host's cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import tempfile
    from oracle import Reference
    from memvanta_b200 import gguf
    R = Reference()
    ws, x = q4_inputs()
    threads = cpu_threads()
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "w.gguf")
        gguf.write_single_tensor(p, "blk.0.attn_q.weight", gguf.Q4_0, Q4_ROWS, Q4_COLS, ws[0])
        h = R.open(p)
        try:
            R.matvec(h, "blk.0.attn_q.weight", x, Q4_ROWS, threads=threads)
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < seconds:
                R.matvec(h, "blk.0.attn_q.weight", x, Q4_ROWS, threads=threads)
                n += 1
            dt = (time.perf_counter() - t0) / n
        finally:
            R.close(h)
    return {"value": Q4_ALG_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{n} tensor_matvec calls on one 4096x4096 Q4_0 weight (oracle/_ref, {threads} threads)"}


# -------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="q4_gemv", choices=["q4_gemv"])
    ap.add_argument("--clock-window", type=float, default=0.5)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    metric, unit = "Q4_0 GEMV achieved HBM GB/s (config 0, 4096x4096)", "GB/s"
    config = {"workload": "config0: Q4_0xQ8 GEMV 4096x4096, x~N(0,1), 32 rotated weight copies (303 MB > 126 MB L2)",
              "rows": Q4_ROWS, "cols": Q4_COLS, "l2": "inputs rotated across 32 weight copies (303 MB, 2.4x L2)",
              "parallelism": f"replicas x{world}"}

    if args.impl == "reference":
        if rank != 0:
            return
        cpu = run_q4_gemv_cpu(seconds=max(2.0, min(20.0, 0.05 * args.steps)))
        line = {"impl": "reference", "metric": metric, "value": cpu["value"], "unit": unit, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "u8",
                "data": "synthetic", "config": config, "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    r = run_q4_gemv_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    peaks = measured_peaks()
    cpu = run_q4_gemv_cpu(seconds=10.0) if world == 1 else None
    value = r["gbs"] * world
    line = {
        "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_total"] / args.steps, "launches_per_step": Q4_COPIES,
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": config,
        "roofline": {"bound": "hbm", "achieved": round(r["gbs"], 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(r["gbs"] / peaks["hbm_gbs"], 4), "traffic": traffic_from_profiles("gemv_q4"),
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": Q4_ALG_BYTES},
        "e2e": {"value": round(r["e2e_gbs"] * world, 3), "unit": unit, "h2d_bytes_per_step": Q4_COLS * 4,
                "d2h_bytes_per_step": Q4_ROWS * 4,
                "path": "mv_tensor_matvec_host (host x/y, H2D + GEMV + D2H + sync per call)"},
        "cpu_baseline": cpu, "clocks": r["clocks"], "gpu_launches": r["gpu_launches"],
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
