#!/usr/bin/env python3
"""Benchmark driver (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads:
  llama7b   config 3 (default) -- random-init OpenLLaMA-7B-shaped Q4_0 Llama
            (Q6_K head), F16 paged KV, ctx 768.  One step = one greedy decode
            token; the K timed steps run from position 128 after a 128-token
            seed prefill, so K = 128 is the reference's tg128.  pp512 (prefill
            batch 32) is timed in the same run and reported beside it.
  q4_gemv   config 0 -- one step = 32 Q4_0 x Q8 GEMVs, one over each of 32
            copies of a 4096x4096 weight (303 MB, 2.4x the 126 MB L2, so every
            launch streams its weight from HBM), metric HBM GB/s.

--clock-window S keeps the same CUDA graph running for S seconds right
before the timed region so nvidia-smi has samples under load (the timed
region itself is unchanged).

Multi-GPU: one process per GPU under torchrun.  llama7b runs ONE model
split over the N GPUs by tensor parallelism (LlamaModel.tensor_parallel:
q/k/v heads, o / gate / up / down / head rows sharded, activations
all-gathered over NVLink peer memory inside the kernels), so the work is
fixed as N grows ("scaling": "strong") and `value` is the one sequence's
tok/s.  q4_gemv runs a replica per rank ("weak"; `value` sums the ranks).
Timing is the max over ranks in both.

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


# ------------------------------------------------------ llama7b (config 3)

L7_PATH = os.environ.get("MV_BENCH_GGUF", "/tmp/memvanta_b200_rand7b_seed1234.gguf")
L7_CTX, L7_SEED_TOKENS, L7_PP, L7_BATCH = 768, 128, 512, 32
# bytes one decode token reads: every Q4_0 layer weight and the Q6_K head once
L7_LAYER_W = 4 * 4096 * 4096 // 32 * 18 + 3 * 11008 * 4096 // 32 * 18
L7_HEAD_W = 32000 * 4096 // 256 * 210


def fixed_tokens(n, vocab=32000, offset=0):
    """The reference bench's prompt ids, (i*1543+17) % vocab
    (benchmarks/real_model_bench.cpp:18)."""
    return ((np.arange(offset, offset + n) * 1543 + 17) % vocab).astype(np.int32)


def ensure_llama7b():
    from memvanta_b200 import gguf
    if not os.path.exists(L7_PATH):
        tmp = L7_PATH + f".tmp{os.getpid()}"
        gguf.write_random_llama(tmp, gguf.LLAMA_7B, seed=1234)
        os.replace(tmp, L7_PATH)
    return L7_PATH


def gemv_roofline(dev, stream, world=1):
    """Live timing of the decode GEMV (the dominant kernel) on the four decode
    shapes, weighted as one token uses them: per layer q|k|v 12288x4096,
    o 4096x4096, gate|up 22016x4096 (SiLU pairs), down 4096x11008 -- each
    rank's share of the rows under tensor parallelism over `world` GPUs."""
    import torch
    import memvanta_b200 as mv
    from memvanta_b200 import gguf
    rng = np.random.default_rng(7)
    total_bytes, total_s, detail = 0, 0.0, {}
    shapes = [("qkv", 12288, 4096), ("o", 4096, 4096), ("gate_up", 22016, 4096), ("down", 4096, 11008)]
    for name, rows, cols in [(n, r // world, c) for n, r, c in shapes]:
        copies = max(2, int(np.ceil(3 * 126e6 / (rows * cols / 32 * 18))))  # > L2 in total
        ws = [mv.Weight.upload(gguf.gen_q4_0(rows, cols, rng), mv.Q4_0, rows, cols) for _ in range(copies)]
        x = torch.randn(cols, device=dev)
        y = torch.empty(rows, device=dev)
        n = 8 * copies
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            mv.gemv(ws[0], x, y, stream)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    mv.gemv(ws[i % copies], x, y, stream)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        per = e0.elapsed_time(e1) / 1e3 / n
        alg = rows * cols // 32 * 18 + cols * 4 + rows * 4
        detail[name] = {"rows": rows, "cols": cols, "us_per_launch": round(per * 1e6, 2),
                        "gbs": round(alg / per / 1e9, 1)}
        total_bytes += alg
        total_s += per
        for w in ws:
            w.free()
        del g
    return total_bytes / total_s / 1e9, total_bytes, total_s, detail


def run_llama7b_ours(args, world, rank, local):
    import torch
    import memvanta_b200 as mv
    mv.init(local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    path = ensure_llama7b()
    t_load = time.perf_counter()
    if world > 1:  # one model over all ranks (tensor parallel, exact)
        m = mv.LlamaModel.tensor_parallel(path, device=local, ctx_override=L7_CTX, kv_page_tokens=16,
                                          kv_type=mv.KV_F16, prefill_batch=L7_PP)  # room for merged batches
    else:
        m = mv.LlamaModel(path, ctx_override=L7_CTX, kv_page_tokens=16, kv_type=mv.KV_F16)
    load_s = time.perf_counter() - t_load  # GGUF parse + upload pipeline (+ peer connect at N > 1)
    ms = torch.cuda.ExternalStream(m.stream)
    K, W = args.steps, args.warmup
    if L7_SEED_TOKENS + max(K, W) > L7_CTX:
        raise SystemExit(f"--steps/--warmup above {L7_CTX - L7_SEED_TOKENS} exceed the ctx {L7_CTX} run")
    seed = fixed_tokens(L7_SEED_TOKENS)
    # warm-up: a full sequence of W decode steps (graphs, clocks, caches)
    m.reset()
    m.prefill(seed, L7_BATCH, False)
    m.generate_greedy(17, W)
    # timed: K greedy decode steps from position 128 (tg128 when K = 128)
    m.reset()
    m.prefill(seed, L7_BATCH, False)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(ms)
        toks = m.generate_greedy(17, K)
        e1.record(ms)
        torch.cuda.synchronize()
    tg_ms = e0.elapsed_time(e1)
    tg_ms = all_max(tg_ms, world)
    # pp512: prefill of the 512-token prompt in batches of 32, one timed call
    prompt = fixed_tokens(L7_PP)
    m.reset()
    m.prefill(prompt, L7_BATCH, True)  # warm-up: buffers and kernels of the 512-token batch
    m.reset()
    torch.cuda.synchronize()
    barrier(world)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(ms)
    m.prefill(prompt, L7_BATCH, True)
    p1.record(ms)
    torch.cuda.synchronize()
    pp_ms = all_max(p0.elapsed_time(p1), world)
    # e2e: the reference contract -- forward(token) returns host logits, the
    # caller samples greedily on the host (real_model_bench tg loop)
    m.reset()
    m.prefill(seed, L7_BATCH, False)
    for _ in range(3):
        m.forward(17)
    m.reset()
    m.prefill(seed, L7_BATCH, False)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    cur, e2e_toks = 17, []
    for _ in range(K):
        cur = int(np.argmax(m.forward(cur)))
        e2e_toks.append(cur)
    e2e_s = all_max(time.perf_counter() - t0, world)
    # the timed device-side greedy loop and the host-argmax forward loop
    # decode the same sequence from the same state: their tokens must agree
    if [int(t) for t in toks] != e2e_toks:
        raise RuntimeError(f"generate_greedy tokens {list(toks[:8])} differ from the forward loop's {e2e_toks[:8]}")
    # embed; per layer q|k|v GEMV, fused RoPE+append+attention, o, gate|up, down;
    # output RMSNorm + Q6_K head GEMV + greedy step; tensor parallel adds the
    # wait before the head, the logits scatter, its wait and the step counter
    kernels_per_step = 1 + 5 * m.n_layer + 3 + (4 if world > 1 else 0)
    batched = run_batched_decode(m, seed) if world == 1 else None
    m.close()
    gbs, alg_bytes, gemv_s, detail = gemv_roofline(dev, torch.cuda.Stream(device=dev), world)
    return {"tg_ms": tg_ms, "pp_ms": pp_ms, "e2e_s": e2e_s, "clocks": clk.summary(), "load_s": load_s,
            "gpu_launches": K * kernels_per_step + 1, "first_tokens": [int(t) for t in toks[:8]],
            "distinct_tokens": len(set(int(t) for t in toks)), "gemv_gbs": gbs, "gemv_detail": detail,
            "batched": batched}


def run_batched_decode(m, seed, n_seq=64, steps=16, warmup=2):
    """Several sequences decoded as one batch (mv_model_forward_batch): n_seq
    sequences, each prefilled with a rotation of the 128-token seed, then
    `steps` batched decode steps, each returning [n_seq, vocab] host logits
    (their device-to-host copy inside the timed region).  Aggregate tok/s."""
    import torch
    S = m.open_sequences(n_seq, L7_SEED_TOKENS + warmup + steps)
    try:
        for i in range(n_seq):
            S.prefill(i, np.roll(seed, i), L7_BATCH, False)
        cur = np.array([(17 + 31 * i) % 32000 for i in range(n_seq)], np.int32)
        for _ in range(warmup):
            cur = np.argmax(S.forward(cur), axis=1).astype(np.int32)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            cur = np.argmax(S.forward(cur), axis=1).astype(np.int32)
        dt = time.perf_counter() - t0
    finally:
        S.close()
    return {"n_seq": n_seq, "steps": steps, "tok_s": round(n_seq * steps / dt, 1),
            "ms_per_step": round(dt / steps * 1e3, 3),
            "ctx": f"{L7_SEED_TOKENS + warmup}..{L7_SEED_TOKENS + warmup + steps} per sequence",
            "timing": "host wall clock around forward_batch calls (logits D2H and host argmax included)",
            "d2h_bytes_per_step": n_seq * 32000 * 4}


def other_configs():
    """BASELINE.json configs 0, 1, 2 and 4 on this GPU, one live timing each
    (time_matmul / time_paged_attn): the headline line carries them as
    extra keys."""
    out = {}
    c0 = time_matmul("gemv", "q4_0", 4096, 4096)
    out["config0_q4_0_gemv_4096x4096"] = {"us": c0["us_per_launch"], "gbs": c0["value"], "hbm_frac": c0["hbm_frac"]}
    c1 = {}
    for name, rows, cols in (("gate_11008x4096", 11008, 4096), ("down_4096x11008", 4096, 11008)):
        for B in (32, 128, 512):
            r = time_matmul("gemm", "q4_0", rows, cols, B)
            c1[f"{name}_b{B}"] = {"us": r["us_per_launch"], "tops": r["value"],
                                  "int8_frac_of_nominal": r["int8_frac_of_nominal"],
                                  "weight_stream_gbs": r["weight_stream_gbs"], "hbm_frac": r["hbm_frac"]}
    out["config1_q4_0_gemm"] = c1
    out["config1_int8_peak_tops"] = {"value": INT8_NOMINAL_TOPS, "source": "nominal dense int8 (no measured figure)"}
    c2 = {}
    for name, wt, rows in (("q8_0_4096x4096", "q8_0", 4096), ("q6_k_32000x4096", "q6_k", 32000)):
        r = time_matmul("gemv", wt, rows, 4096)
        c2[f"{name}_b1"] = {"us": r["us_per_launch"], "gbs": r["value"], "hbm_frac": r["hbm_frac"]}
        r = time_matmul("gemm", wt, rows, 4096, 32)
        c2[f"{name}_b32"] = {"us": r["us_per_launch"], "weight_stream_gbs": r["weight_stream_gbs"],
                             "hbm_frac": r["hbm_frac"]}
    out["config2_mixed_quant"] = c2
    c4 = {}
    for kv in ("f16", "q8_0"):
        for split in (True, False):
            r = time_paged_attn(kv, split=split)
            c4[kv + ("_split_k" if split else "_exact")] = {"us": r["us_per_launch"], "gbs": r["value"],
                                                            "hbm_frac": r["frac_of_measured_hbm"],
                                                            "sum_ctx": r["sum_ctx"]}
    out["config4_paged_attention"] = c4
    return out


def run_llama7b_cpu(threads=None, prompt=512, gen=16):
    """The reference's own memvanta_real_bench (oracle/_ref, built from the
    unmodified sources) on this host's cores: pp<prompt> and tg<gen> tok/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import REF_REAL_BENCH
    path = ensure_llama7b()
    threads = threads or cpu_threads()
    cmd = [REF_REAL_BENCH, "--model", path, "--threads", str(threads), "--ctx", str(L7_CTX), "--prompt", str(prompt),
           "--gen", str(gen), "--batch", str(L7_BATCH), "--kv", "f16", "--warmup", "0", "--reps", "1", "--no-client"]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    if out.returncode != 0:
        raise RuntimeError(f"reference bench failed: {out.stderr.strip()[-300:]}")
    vals = {}
    for line in out.stdout.splitlines():
        parts = [p.strip() for p in line.split("|")]
        if len(parts) > 7 and (parts[6].startswith("pp") or parts[6].startswith("tg")):
            vals[parts[6][:2]] = float(parts[7].split()[0])
    return {"tg": vals.get("tg"), "pp": vals.get("pp"), "threads": threads,
            "sample": f"memvanta_real_bench --prompt {prompt} --gen {gen} --batch {L7_BATCH} --ctx {L7_CTX} --kv f16 "
                      f"--threads {threads} on the same random 7B GGUF (tg after a 128-token seed prefill)"}


# -------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="llama7b",
                    choices=["llama7b", "q4_gemv", "gemv", "gemm", "decode", "prefill", "paged_attn"],
                    help="llama7b: the headline (config 3); q4_gemv: config 0; gemv / gemm / decode / prefill: "
                         "one kernel, or the 7B decode steps or pp512 prefill alone, for profiling")
    ap.add_argument("--rows", type=int, default=12288, help="gemv/gemm: weight rows")
    ap.add_argument("--cols", type=int, default=4096, help="gemv/gemm: weight cols (K)")
    ap.add_argument("--batch", type=int, default=32, help="gemm: tokens")
    ap.add_argument("--wtype", default="q4_0", choices=["q4_0", "q8_0", "q6_k"],
                    help="gemv/gemm: weight type (config 2: q8_0 4096x4096, q6_k 32000x4096; the gemm of q8_0 and "
                         "q6_k runs the reference's fp32-activation path)")
    ap.add_argument("--kv", default="f16", choices=["f16", "q8_0"], help="paged_attn: cache type")
    ap.add_argument("--attn", default="split", choices=["split", "exact"],
                    help="paged_attn: split-K kernel or the exact-order kernel")
    ap.add_argument("--clock-window", type=float, default=0.5)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.workload in ("gemv", "gemm", "decode", "prefill", "paged_attn"):
        return main_micro(args)
    if args.workload == "llama7b":
        return main_llama7b(args, world, rank, local)
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


def main_micro(args):
    """One kernel (or the 7B decode steps alone) on one GPU, for profiling:
    gemv = the decode GEMV on a rows x cols Q4_0 weight (activations
    quantised per call), gemm = Q8 quantisation + the tensor-core GEMM for
    `batch` tokens, decode = `steps` greedy decode steps of the 7B model after
    its 128-token seed prefill.  Weights rotate through copies larger than L2;
    launches are replayed from a CUDA graph and timed with events."""
    import torch
    import memvanta_b200 as mv
    from memvanta_b200 import gguf
    mv.init(0)
    dev = torch.device("cuda", 0)
    if args.workload == "decode":
        m = mv.LlamaModel(ensure_llama7b(), ctx_override=L7_CTX, kv_page_tokens=16, kv_type=mv.KV_F16)
        ms = torch.cuda.ExternalStream(m.stream)
        seed = fixed_tokens(L7_SEED_TOKENS)
        m.prefill(seed, L7_BATCH, False)
        m.generate_greedy(17, args.warmup)
        m.reset()
        m.prefill(seed, L7_BATCH, False)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(ms)
        m.generate_greedy(17, args.steps)
        e1.record(ms)
        torch.cuda.synchronize()
        ms_step = e0.elapsed_time(e1) / args.steps
        m.close()
        print(json.dumps({"workload": "decode", "metric": "7B Q4_0 decode tok/s", "value": round(1e3 / ms_step, 2),
                          "unit": "tok/s", "ms_per_step": round(ms_step, 4), "steps": args.steps}), flush=True)
        return
    if args.workload == "prefill":
        # pp512 alone: `steps` prefills of the 512-token prompt in batches of
        # 32 after one warm-up prefill of the same prompt
        m = mv.LlamaModel(ensure_llama7b(), ctx_override=L7_CTX, kv_page_tokens=16, kv_type=mv.KV_F16)
        ms = torch.cuda.ExternalStream(m.stream)
        prompt = fixed_tokens(L7_PP)
        m.prefill(prompt, L7_BATCH, True)  # warm-up: the 512-token batch's buffers and kernels
        total = 0.0
        for _ in range(args.steps):
            m.reset()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(ms)
            m.prefill(prompt, L7_BATCH, True)
            e1.record(ms)
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        m.close()
        ms_pp = total / args.steps
        print(json.dumps({"workload": "prefill", "metric": "7B Q4_0 pp512 tok/s", "value": round(L7_PP / ms_pp * 1e3, 2),
                          "unit": "tok/s", "ms_per_prefill": round(ms_pp, 3), "steps": args.steps}), flush=True)
        return
    if args.workload == "paged_attn":
        return main_paged_attn(args, mv, dev)
    line = time_matmul(args.workload, args.wtype, args.rows, args.cols, args.batch, args.steps, args.warmup)
    print(json.dumps(line), flush=True)


INT8_NOMINAL_TOPS = 4500.0  # dense int8 tensor peak, nominal (NVIDIA's figure without sparsity)


def time_matmul(kind, wtype, rows, cols, B=1, steps=32, warmup=3):
    """Live time of one decode GEMV (kind "gemv") or batched matmul ("gemm":
    Q8 quantisation of X included, tensor_matmul_batch_v06's dispatch) on a
    rows x cols weight of `wtype`.  Weights rotate through copies larger than
    3x L2; launches are replayed from a CUDA graph and timed with events on
    the launching stream."""
    import torch
    import memvanta_b200 as mv
    from memvanta_b200 import gguf
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(7)
    wt = {"q4_0": gguf.Q4_0, "q8_0": gguf.Q8_0, "q6_k": gguf.Q6_K}[wtype]
    wbytes = gguf.tensor_nbytes(wt, rows * cols)
    copies = max(2, int(np.ceil(3 * 126e6 / wbytes)))
    ws = [mv.Weight.upload(gguf.gen_blocks(wt, rows, cols, rng), wt, rows, cols) for _ in range(copies)]
    act = mv.ACT_Q8 if wt == gguf.Q4_0 else mv.ACT_F32  # tensor_matmul_batch_v06's dispatch
    n = max(steps, copies)
    stream = torch.cuda.Stream(device=dev)
    if kind == "gemv":
        x, y = torch.randn(cols, device=dev), torch.empty(rows, device=dev)
        launch = lambda w: mv.gemv(w, x, y, stream)  # noqa: E731
    else:
        x, y = torch.randn(B, cols, device=dev), torch.empty(B, rows, device=dev)
        launch = lambda w: mv.gemm(w, x, y, act, stream)  # noqa: E731
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 1)):
            launch(ws[i % copies])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                launch(ws[i % copies])
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    mv.stream_status(stream)
    us = e0.elapsed_time(e1) * 1e3 / n
    del g
    for w in ws:
        w.free()
    line = {"workload": kind, "wtype": wtype, "rows": rows, "cols": cols, "us_per_launch": round(us, 3),
            "launches": n}
    peak = measured_peaks()["hbm_gbs"]
    if kind == "gemv":
        alg = wbytes + cols * 4 + rows * 4
        line.update({"metric": f"{wtype} GEMV achieved GB/s", "value": round(alg / us / 1e3, 1), "unit": "GB/s",
                     "algorithmic_bytes_per_launch": alg, "hbm_frac": round(alg / us / 1e3 / peak, 4)})
    else:
        alg = wbytes + B * cols * 4 + B * rows * 4
        tops = 2 * rows * cols * B / us / 1e6
        line.update({"batch": B, "metric": f"{wtype} GEMM TOPS (2*rows*cols*batch / time"
                                           + (", Q8 quantisation included)" if wt == gguf.Q4_0 else ", fp32 x)"),
                     "value": round(tops, 2), "unit": "TOPS",
                     "weight_stream_gbs": round(alg / us / 1e3, 1), "hbm_frac": round(alg / us / 1e3 / peak, 4)})
        if wt == gguf.Q4_0:
            line["int8_frac_of_nominal"] = round(tops / INT8_NOMINAL_TOPS, 4)
    return line


def main_paged_attn(args, mv, dev):
    print(json.dumps(time_paged_attn(args.kv, args.steps, args.warmup, args.attn == "split")), flush=True)


def time_paged_attn(kv="f16", steps=32, warmup=3, split=True):
    """Config 4: paged decode attention over 64 sequences, ctx ~ U(64..768),
    16-token pages scattered by a random permutation block table, 32 heads x
    128, Q/K/V ~ N(0,1) (random fp16 pages; Q8_0 pages with random int8 and
    scales for --kv q8_0).  The cache (~436 MB F16) is larger than L2, so every
    launch reads it from HBM.  One launch per step, replayed from a graph."""
    import torch
    import memvanta_b200 as mv
    dev = torch.device("cuda", torch.cuda.current_device())
    kv_type = {"f16": mv.KV_F16, "q8_0": mv.KV_Q8_0}[kv]
    rng = np.random.default_rng(4)
    n_seq, n_head, hd, page = 64, 32, 128, 16
    kv_dim = n_head * hd
    ctx = rng.integers(64, 769, n_seq).astype(np.int32)
    max_pages = int((ctx.max() + page - 1) // page)
    npg = (ctx + page - 1) // page
    total = int(npg.sum())
    perm = rng.permutation(total).astype(np.int32)
    table = np.zeros((n_seq, max_pages), np.int32)
    o = 0
    for s_ in range(n_seq):
        table[s_, :npg[s_]] = perm[o:o + npg[s_]]
        o += npg[s_]
    slots = total * page
    g = torch.Generator(device=dev).manual_seed(4)
    if kv_type == mv.KV_F16:
        kp = torch.randn((slots, kv_dim), generator=g, device=dev).half().view(torch.uint8)
        vp = torch.randn((slots, kv_dim), generator=g, device=dev).half().view(torch.uint8)
        ks = vs = None
    else:
        kp = torch.randint(-127, 128, (slots, kv_dim), generator=g, device=dev, dtype=torch.int8).view(torch.uint8)
        vp = torch.randint(-127, 128, (slots, kv_dim), generator=g, device=dev, dtype=torch.int8).view(torch.uint8)
        ks = torch.rand((slots, kv_dim // 32), generator=g, device=dev) * 0.02
        vs = torch.rand((slots, kv_dim // 32), generator=g, device=dev) * 0.02
    q = torch.randn((n_seq, kv_dim), generator=g, device=dev)
    tab, ctx_t = torch.from_numpy(table).to(dev), torch.from_numpy(ctx).to(dev)
    out = torch.empty((n_seq, kv_dim), device=dev)
    stream = torch.cuda.Stream(device=dev)
    fn = mv.paged_attn_decode_split if split else mv.paged_attn_decode
    call = lambda: fn(kv_type, q, n_head, n_head, hd, kp, vp, tab, max_pages, page, ctx_t,  # noqa: E731
                      int(ctx.max()), ks, vs, out, stream)
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 1)):
            call()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(steps):
                call()
        gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        gr.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    del gr
    row_bytes = mv.kv_row_bytes(kv_type, kv_dim) + 4 * mv.kv_row_scales(kv_type, kv_dim)
    alg = int(ctx.sum()) * 2 * row_bytes + 2 * n_seq * kv_dim * 4  # K and V of every context token, Q in, O out
    return {"workload": "paged_attn", "kv": kv, "kernel": "split-K" if split else "exact order",
            "config": "config4: 64 seqs, ctx U(64..768), 16-token "
            "pages, random permutation block table, 32 heads x 128", "sum_ctx": int(ctx.sum()),
            "us_per_launch": round(us, 2), "metric": "paged attention achieved GB/s",
            "value": round(alg / us / 1e3, 1), "unit": "GB/s", "algorithmic_bytes_per_launch": alg,
            "frac_of_measured_hbm": round(alg / us / 1e3 / measured_peaks()["hbm_gbs"], 3)}


def main_llama7b(args, world, rank, local):
    metric, unit = "7B Q4_0 tg128 tok/s", "tok/s"
    config = {"workload": f"config3: random-init OpenLLaMA-7B-shaped Llama, Q4_0 layers + Q6_K head, F16 paged KV "
                          f"(16-token pages), ctx {L7_CTX}; {args.steps} greedy decode tokens from position "
                          f"{L7_SEED_TOKENS}; pp512 = 512-token prompt prefilled in batches of {L7_BATCH}",
              "model": "llama-7b-shape (32L, d4096, 32h x 128, ffn 11008, vocab 32000)",
              "global_batch": 1, "seq_len": L7_CTX,
              "parallelism": f"tp{world} (exact all-gather tensor parallel)" if world > 1 else "single GPU",
              "l2": "decode reads 3.75 GB of weights per token (30x the 126 MB L2)"}
    if args.impl == "reference":
        if rank != 0:
            return
        # the same workload as our arm: pp512 in batches of 32, then K = --steps
        # greedy decode tokens after the reference bench's 128-token seed prefill
        cpu = run_llama7b_cpu(prompt=L7_PP, gen=args.steps)
        line = {"impl": "reference", "metric": metric, "value": cpu["tg"], "unit": unit, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "q4_0/q8",
                "data": "synthetic", "config": config, "pp_tok_s": cpu["pp"],
                "cpu_baseline": {"value": cpu["tg"], "unit": unit, "cores": cpu["threads"], "kind": "reference",
                                 "sample": cpu["sample"]},
                "e2e": {"value": cpu["tg"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    r = run_llama7b_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    extra = other_configs() if world == 1 else {}
    peaks = measured_peaks()
    cpu = None
    if world == 1:
        c = run_llama7b_cpu()
        cpu = {"value": c["tg"], "unit": unit, "cores": c["threads"], "kind": "reference", "sample": c["sample"],
               "pp_tok_s": c["pp"]}
    tg = args.steps / (r["tg_ms"] / 1e3)
    pp = L7_PP / (r["pp_ms"] / 1e3)
    bytes_per_token = 32 * L7_LAYER_W + L7_HEAD_W
    qkv = r["gemv_detail"]["qkv"]
    qkv_alg = qkv["rows"] * qkv["cols"] // 32 * 18 + qkv["cols"] * 4 + qkv["rows"] * 4
    line = {
        "metric": metric, "value": round(tg, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["tg_ms"] / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_0 x q8 (int8 dot, fp32 accumulate)",
        "data": "synthetic (random-init weights, seeded)", "config": config,
        "pp512_tok_s": round(pp, 2), "pp512_ms": round(r["pp_ms"], 2), "model_load_s": round(r["load_s"], 2),
        "decode_weight_bw_gbs": round(bytes_per_token * tg / 1e9, 1),
        # the dominant decode kernel, one launch of its q|k|v shape: live
        # algorithmic bytes / live time; traffic = ncu DRAM bytes of the same launch
        "roofline": {"bound": "hbm",
                     "kernel": f"mvb::gemv_q4_tile_kernel (Q4_0 x Q8 decode GEMV), q|k|v {qkv['rows']}x{qkv['cols']} "
                               f"launch (one rank's share)",
                     "achieved": qkv["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(qkv["gbs"] / peaks["hbm_gbs"], 4),
                     "traffic": traffic_from_profiles("gemv_q4_qkv") if world == 1 else None,
                     "algorithmic_bytes_per_launch": qkv_alg,
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, burst)",
                     "all_shapes_weighted_gbs": round(r["gemv_gbs"], 1), "shapes": r["gemv_detail"]},
        "e2e": {"value": round(args.steps / r["e2e_s"], 2), "unit": unit, "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 32000 * 4,
                "path": "LlamaModel.forward (mv_model_forward): token in, host logits out, host argmax per token"},
        "cpu_baseline": cpu, "clocks": r["clocks"], "gpu_launches": r["gpu_launches"],
        "first_tokens": r["first_tokens"], "distinct_tokens": r["distinct_tokens"],
        "greedy_check": "generate_greedy tokens == forward-loop (host argmax) tokens",
    }
    if r.get("batched"):
        line["batched_decode_64_sequences"] = r["batched"]
    line.update(extra)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
