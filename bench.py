#!/usr/bin/env python
"""Decode-throughput benchmark (one JSON line on rank 0).

Workload: Llama-3-8B-shape random-init model, Q4_0
(dim 4096, 32 layers, 32/8 heads, FFN 14336, vocab 128256), greedy decode at
batch 1 with an f16 KV cache holding 4096 positions.  A step is one decoded
token.  Weights stream from HBM every step (4.2 GB >> the 126 MB L2).

  value   tok/s of the device-resident decode loop (the per-token CUDA graph
          replayed back to back, sampled id fed back on the device)
  e2e     tok/s through the C ABI per token: host token id in (H2D), sampled
          id out (D2H), prana_forward per step
  roofline  the Q4_0 GEMV at the gate|up shape [28672 x 4096], rotating weight
          copies larger than L2, timed in a CUDA graph with events on its stream
  cpu_baseline  the CPU oracle (C restatement of Prana's AVX2/VNNI path and
          worker pool) decoding the same model from the same KV contents
  batch_decode  (one GPU) batch 16: 16 independent sequences with their own KV
          caches at the same context, one token each per prana_forward_multi
          call, host ids in and out (the BASELINE config's bs 16)

Both arms start from the same seeded KV contents (4096 rows of N(0, 0.5) f16
per layer) instead of a 4096-token prefill, so the CPU arm finishes in minutes;
the bytes a decode step reads are the same either way.

--gpus N > 1 (under torchrun): the model is tensor-parallel over the N GPUs
(column-split Q/K/V and gate|up, row-split wo and ffn_down, vocabulary-split
LM head; a one-shot all-reduce over NVLink peer memory after wo and after
ffn_down), one sequence, so the work per token is fixed (strong scaling);
value is that sequence's tok/s.
--impl reference: the CPU oracle alone on the host cores (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import threading
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s at batch 1"
UNIT = "tok/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=512)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", default="prana", choices=["prana", "reference"])
    p.add_argument("--workload", default="llama3_8b_q4_0")
    p.add_argument("--ctx", type=int, default=4096)
    p.add_argument("--model-dir", default=os.environ.get("PRANA_BENCH_DIR", "/dev/shm/prana_bench"))
    p.add_argument("--cpu-seconds", type=float, default=20.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--batch-seqs", type=int, default=16,
                   help="also time this many independent sequences per step (0: skip; single GPU only)")
    return p.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def model_path(args, rank):
    from prana_b200 import synth

    spec = synth.PRESETS[args.workload]
    d = Path(args.model_dir)
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"{args.workload}_seed{spec.seed}.gguf"
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(".tmp")
        synth.write_gguf(spec, tmp)
        tmp.rename(path)
    return spec, path


def seeded_kv_rows(layer, is_v, rows, kv_dim, seed=4242):
    rng = np.random.default_rng([seed, layer, int(is_v)])
    return (rng.standard_normal((rows, kv_dim), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)


def launches_per_step(spec, world=1, peer=False) -> int:
    """Kernels of this library per decode step (NCCL's own kernels not counted;
    the peer-memory exchange adds 2 all-reduces per layer and the argmax
    all-gather)."""
    types = [spec.type_q, spec.type_k, spec.type_v]
    qkv = 1 + sum(1 for i in range(1, 3) if types[i] != types[i - 1])
    swiglu = 1 if spec.type_gate == spec.type_up else 4
    # embed + per layer (qkv, attention, wo, ffn, down) + lm head (+ the cross-rank argmax) + advance
    n = 1 + spec.n_layers * (qkv + 1 + 1 + swiglu + 1) + 1 + (1 if world > 1 else 0) + 1
    if world > 1 and peer:
        n += 2 * spec.n_layers + 1
    return n


class Clocks:
    """nvidia-smi samples (every 100 ms) kept only when they fall inside the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.reader = None

    def start(self):
        """Start sampling; returns once the first sample is in, so the region that follows is covered."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                self.lines.append((time.monotonic(), line))

        self.reader = threading.Thread(target=read, daemon=True)
        self.reader.start()
        t_end = time.monotonic() + 10.0
        while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
            time.sleep(0.02)

    def stop(self, t0, t1):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.reader.join(timeout=5)
        inside = [ln for ts, ln in self.lines if t0 <= ts <= t1]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in inside:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_decode(path, ctx, kv_rows_fn, n_layers, kv_dim, seconds, token=17, max_steps=None):
    """Time the CPU oracle decoding from `ctx` with the given KV rows; returns (tok/s, steps, threads)."""
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    orc.lib().or_pool_set_threads(threads)
    om = orc.OModel(str(path), orc.TIER_AUTO)
    kv = om.kv(ctx + 64)
    for layer in range(n_layers):
        for is_v in (False, True):
            kv.set_layer(layer, is_v, kv_rows_fn(layer, is_v))
    om.forward(kv, token, ctx)  # warm the pool and caches
    t0 = time.perf_counter()
    steps, pos, tok = 0, ctx + 1, token
    while True:
        lg = om.forward(kv, tok, pos)
        tok = int(np.argmax(lg))
        steps += 1
        pos += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_steps and steps >= max_steps) or pos >= ctx + 60:
            break
    tier = {1: "scalar", 2: "avx2", 3: "vnni"}[orc.lib().or_default_tier()]
    return steps / el, steps, threads, tier, el


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from prana_b200 import synth

    spec, path = model_path(args, 0)
    kv_dim = spec.n_kv_heads * spec.head_dim
    budget = max(30.0, min(150.0, (args.steps + args.warmup) * 2.0))
    tps, steps, threads, tier, el = cpu_decode(path, args.ctx, lambda l, v: seeded_kv_rows(l, v, args.ctx, kv_dim),
                                               spec.n_layers, kv_dim, budget, max_steps=args.steps)
    sample = (f"{steps} greedy decode tokens at positions {args.ctx + 1}.. from seeded KV ({args.workload}), "
              f"{threads} threads, {tier} tier, {el:.1f} s; C restatement of Prana's CPU path (Rust toolchain absent)")
    line = {"metric": METRIC, "value": round(tps, 4), "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": 1, "ms_per_step": round(1000.0 / tps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> int32 / f32", "data": "synthetic",
            "config": {"workload": args.workload, "ctx": args.ctx, "batch": 1},
            "cpu_baseline": {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(tps, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) per launch of the roofline kernel, from one ncu --set full
# capture of this same launch (mean of launches 1 and 2: 66.91 and 66.62 MB); the
# command and the figures are in profiles/stream_gemv_q4_0_llama3_8b.txt.
ROOFLINE_TRAFFIC = 66_764_000
ROOFLINE_TRAFFIC_SOURCE = "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/stream_gemv_q4_0_llama3_8b.txt"


def gemv_roofline(torch, peak_gbs, iters=64):
    """Q4_0 GEMV [28672 x 4096] at batch 1: the shape of the fused gate|up weight, the step's largest GEMV."""
    from prana_b200 import kernels as K
    from prana_b200 import synth
    from prana_b200._ffi import TYPE_Q4_0

    rows, cols = 28672, 4096
    raw = synth.matrix(TYPE_Q4_0, rows, cols, seed=77)
    copies = [K.QuantMatrix(TYPE_Q4_0, rows, cols, raw) for _ in range(6)]  # 6 x 66 MB > 3 x L2
    acts = K.quantize_acts(torch.randn(1, cols, device="cuda"))  # int8 rows, as a decode step feeds them
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for w in copies:
            K.matmul_kquant_prefill(acts, w)
    torch.cuda.synchronize()
    # capture the launches so the timing sees the kernel, not Python call overhead
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
        for i in range(iters):
            K.matmul_kquant_prefill(acts, copies[i % len(copies)])
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(side)
    with torch.cuda.stream(side):
        graph.replay()
    e1.record(side)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    alg = rows * cols // 32 * 18 + cols * 4 + rows * 4  # GGUF weight bytes + f32 in + f32 out
    gbs = alg / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(gbs / peak_gbs, 4), "traffic": ROOFLINE_TRAFFIC, "traffic_source": ROOFLINE_TRAFFIC_SOURCE,
            "kernel": "stream_gemv Q4_0 [28672 x 4096] M=1",
            "us_per_launch": round(us, 2), "algorithmic_bytes": alg}


def batch_decode(torch, model, args, stream, steps=24, warmup=3):
    """Decode at batch B = args.batch_seqs: B independent sequences, each with its
    own KV cache at the same context, one token each per prana_forward_multi
    call (host token ids in, host argmax out).  The reference has no
    multi-sequence batch; its equivalent is B forward calls per step."""
    from prana_b200 import model as pm

    c, n = model.config, args.batch_seqs
    caches = [pm.KvCache(model, args.ctx + steps + warmup + 8) for _ in range(n)]
    try:
        for layer in range(c.n_layers):
            for is_v in (False, True):
                rows = seeded_kv_rows(layer, is_v, args.ctx, c.kv_dim())
                for kv in caches:
                    kv.write(layer, is_v, rows)
        toks = (np.arange(n, dtype=np.uint32) * 7919 + 17) % c.vocab_size
        pos = args.ctx
        for _ in range(warmup):
            _, toks = pm.forward_multi(model, caches, toks, [pos] * n, want_logits=False)
            pos += 1
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            _, toks = pm.forward_multi(model, caches, toks, [pos] * n, want_logits=False)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"value": round(n * 1000.0 / ms, 2), "unit": "tok/s", "sequences": n, "ms_per_step": round(ms, 3),
                "steps": steps, "ctx": args.ctx, "h2d_bytes_per_step": 4 * n + 8 * n, "d2h_bytes_per_step": 4 * n,
                "path": "prana_forward_multi: GEMV rows in chunks of 8, attention per sequence"}
    finally:
        for kv in caches:
            kv.close()


def prana_arm(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    torch.cuda.set_device(local)
    from prana_b200 import model as pm

    spec, path = model_path(args, rank)
    tp = None
    if dist:
        dist.barrier()
        # tensor parallel over the ranks: rank 0's NCCL id reaches every rank
        uid = [pm.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = (world, rank, uid[0])
    peak, peak_kind = peaks()
    t_load = time.perf_counter()
    model = pm.Model.load(str(path), local, tp=tp)
    t_load = time.perf_counter() - t_load
    c = model.config
    kv_dim = c.kv_dim()
    kv_l = model.local_kv_dim()  # this rank's kv heads
    cap = args.ctx + 2 * (args.warmup + args.steps) + 16
    kv = pm.KvCache(model, cap)
    for layer in range(c.n_layers):
        for is_v in (False, True):
            rows = seeded_kv_rows(layer, is_v, args.ctx, kv_dim)
            kv.write(layer, is_v, rows[:, rank * kv_l:(rank + 1) * kv_l] if world > 1 else rows)
    stream = torch.cuda.ExternalStream(model.stream())

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- value: device-resident decode loop
    loop = pm.DecodeLoop(model, kv)
    loop.begin(17, args.ctx)
    loop.run(args.warmup)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    t_region = time.monotonic()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    loop.run(args.steps)
    e1.record(stream)
    barrier()
    clk = clocks.stop(t_region, time.monotonic())
    ms = e0.elapsed_time(e1) / args.steps
    toks = loop.tokens(args.warmup + args.steps)
    # ---- e2e: C-ABI call per token with host buffers
    pos = args.ctx + args.warmup + args.steps
    tok = int(toks[-1]) if len(toks) else 17
    for _ in range(args.warmup):
        _, tok = pm.forward(model, kv, tok, pos, want_logits=False)
        pos += 1
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        _, tok = pm.forward(model, kv, tok, pos, want_logits=False)
        pos += 1
    f1.record(stream)
    barrier()
    ms_e2e = f0.elapsed_time(f1) / args.steps
    if dist:
        t = torch.tensor([ms, ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    batch = batch_decode(torch, model, args, stream) if world == 1 and args.batch_seqs > 0 else None
    roof = gemv_roofline(torch, peak) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, steps, threads, tier, el = cpu_decode(path, args.ctx, lambda l, v: seeded_kv_rows(l, v, args.ctx, kv_dim),
                                                   c.n_layers, kv_dim, args.cpu_seconds)
        cpu = {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{steps} greedy tokens at ctx {args.ctx + 1}.. from the same seeded KV, {tier} tier, {el:.1f} s"}
    if rank == 0:
        bytes_tok = spec.weight_bytes_per_token() + 2 * c.n_layers * (args.ctx + args.warmup + args.steps // 2) * kv_dim * 2
        step_gbs = bytes_tok * (1000.0 / ms) / 1e9
        line = {
            "metric": METRIC, "value": round(1000.0 / ms, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> int32 / f32 (Q4_0 weights, f16 KV)",
            "data": "synthetic", "impl": "prana",
            "config": {"workload": args.workload, "ctx": args.ctx, "batch": 1,
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "exchange": ("peer memory" if model.peer_exchange else "nccl") if world > 1 else None,
                       "l2": "inputs larger than L2 (4.2 GB weights per step)"},
            "e2e": {"value": round(1000.0 / ms_e2e, 3), "unit": UNIT, "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4},
            "roofline": roof, "peak_kind": peak_kind,
            "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": round(step_gbs, 1),
                              "frac": round(step_gbs / peak, 4)},
            "cpu_baseline": cpu, "batch_decode": batch, "clocks": clk, "gpu_launches": launches_per_step(spec, world, model.peer_exchange) * args.steps,
            "load_s": round(t_load, 1),
        }
        print(json.dumps(line), flush=True)
    kv.close()
    model.close()
    if dist:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        prana_arm(args)


if __name__ == "__main__":
    main()
