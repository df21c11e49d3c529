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
SAMPLE_TEMP, SAMPLE_SEED = 0.8, 2024  # the sampled-loop line: Sampler::new(0.8, 2024)


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
    p.add_argument("--configs", default=None,
                   help="comma list of the other BASELINE configs to measure in the same line "
                        "(c1,c2,c3,c4q8,c5; default: all on one GPU, none under tensor parallelism)")
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
    """nvidia-smi samples (every 20 ms) kept only when they fall inside the timed region."""

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
                                          "--format=csv,noheader,nounits", "-lms", "20"],
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


def margin(lg) -> float:
    """top-2 logit margin relative to the largest magnitude (the greedy-parity gate)."""
    srt = np.sort(np.asarray(lg, np.float64))
    return float((srt[-1] - srt[-2]) / max(float(np.max(np.abs(lg))), 1e-30))


def forced_parity(path, model, ctx, rows_fn, n_layers, start_tok, gpu_toks, n_steps):
    """The benchmarked token stream, step by step, against the CPU oracle in
    forced mode (oracle/parity.py): the GPU's traced pass replays each step from
    the same seeded cache (it must reproduce the benchmarked token), the oracle
    takes the same step proving every int8 / f16 difference a rounding tie and
    following the GPU's rows; logits must agree within 1e-3 and the token must
    be the oracle's argmax wherever its top-2 margin exceeds 1e-3."""
    from oracle import oracle as orc
    from oracle.parity import Flips, forced_decode, rel
    from prana_b200 import model as pm

    orc.lib().or_pool_set_threads(os.cpu_count() or 1)
    om = orc.OModel(str(path), orc.TIER_AUTO)
    n_steps = min(n_steps, len(gpu_toks))
    okv, gkv = om.kv(ctx + n_steps + 4), pm.KvCache(model, ctx + n_steps + 4)
    try:
        for layer in range(n_layers):
            for is_v in (False, True):
                rows = rows_fn(layer, is_v)
                okv.set_layer(layer, is_v, rows)
                gkv.write(layer, is_v, rows)
        flips = Flips()
        gated = same = replay = 0
        worst = 0.0
        tok = start_tok
        err = None
        for i in range(n_steps):
            try:
                lg_g, lg_o = forced_decode(om, okv, model, gkv, tok, ctx + i, flips, f"step {i}")
            except AssertionError as e:
                err = str(e)
                break
            g = int(np.argmax(lg_g))
            replay += int(g == int(gpu_toks[i]))
            worst = max(worst, rel(lg_g, lg_o))
            if margin(lg_o) > 1e-3:
                gated += 1
                same += int(g == int(np.argmax(lg_o)))
            tok = int(gpu_toks[i])
        out = {"steps": n_steps, "replay_equals_benchmarked": replay, "margin_gated": gated, "identical": same,
               "max_logit_rel_err": float(f"{worst:.3g}"), "int8_tie_flips": flips.flips,
               "int8_compared": flips.total, "f16_kv_tie_flips": flips.kv_flips,
               "rule": "oracle forced with the GPU's int8 rows and f16 K/V rows after each difference is proven "
                       "a rounding tie; logits within 1e-3; identical where the oracle's top-2 margin > 1e-3"}
        if err:
            out["failed"] = err
        return out
    finally:
        gkv.close()


PARITY_RULE = ("CPU oracle fed the GPU's tokens (same seeded KV, same start); a token counts as gated when the "
               "oracle's top-2 margin exceeds 1e-3 of the largest logit, and identical when the GPU chose the "
               "oracle's argmax")


def cpu_decode(path, ctx, kv_rows_fn, n_layers, kv_dim, seconds, token=17, max_steps=None, threads=None,
               follow=None):
    """Time the CPU oracle decoding from position `ctx` after the given KV rows.

    Starts from (token, ctx) like the GPU loop.  With `follow` (the GPU's tokens
    from the same start) the oracle is fed those tokens and each of its argmaxes
    is compared with the GPU's (margin-gated).  Returns (tok/s, steps, threads,
    tier, seconds, parity or None)."""
    from oracle import oracle as orc

    threads = threads or os.cpu_count() or 1
    orc.lib().or_pool_set_threads(threads)
    om = orc.OModel(str(path), orc.TIER_AUTO)
    kv = om.kv(ctx + 64)
    for layer in range(n_layers):
        for is_v in (False, True):
            kv.set_layer(layer, is_v, kv_rows_fn(layer, is_v))
    cmp = gated = same = 0
    steps, pos, tok = 0, ctx, token
    t0 = None
    while True:
        lg = om.forward(kv, tok, pos)
        mine = int(np.argmax(lg))
        if follow is not None and steps < len(follow):
            cmp += 1
            if margin(lg) > 1e-3:
                gated += 1
                same += int(mine == int(follow[steps]))
            tok = int(follow[steps])
        else:
            tok = mine
        steps += 1
        pos += 1
        if t0 is None:  # the first step warms the pool and caches
            t0, steps = time.perf_counter(), 0
            if follow is not None:
                follow = follow[1:]
            continue
        el = time.perf_counter() - t0
        if el >= seconds or (max_steps and steps >= max_steps) or pos >= ctx + 60:
            break
    tier = {1: "scalar", 2: "avx2", 3: "vnni"}[orc.lib().or_default_tier()]
    parity = None
    if follow is not None:
        parity = {"tokens_compared": cmp, "margin_gated": gated, "identical": same, "rule": PARITY_RULE}
    return steps / el, steps, threads, tier, el, parity


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from prana_b200 import synth

    spec, path = model_path(args, 0)
    kv_dim = spec.n_kv_heads * spec.head_dim
    budget = max(30.0, min(150.0, (args.steps + args.warmup) * 2.0))
    tps, steps, threads, tier, el, _ = cpu_decode(path, args.ctx, lambda l, v: seeded_kv_rows(l, v, args.ctx, kv_dim),
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
                "path": "prana_forward_multi, one CUDA graph per cache set: tensor-core GEMMs over the 16 rows, one attention launch over all sequences"}
    finally:
        for kv in caches:
            kv.close()


# ---------------------------------------------------------------- the other BASELINE configs
#
# Each returns one object of the line's "configs": the config's metric measured
# on this GPU through the same public API (value: device-resident loop; e2e:
# host ids in and out), its roofline where one applies, and the CPU oracle on
# a bounded sample of the same workload beside it.


def _preset_path(args, name):
    from prana_b200 import synth

    spec = synth.PRESETS[name]
    d = Path(args.model_dir)
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"{name}_seed{spec.seed}.gguf"
    if not path.exists():
        tmp = path.with_suffix(".tmp")
        synth.write_gguf(spec, tmp)
        tmp.rename(path)
    return spec, path


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def suite_c1(torch, args, peak):
    """C1: stories15M shape, Q8_0: 8 seeded prompt ids, greedy 248 tokens, bs 1."""
    from oracle import oracle as orc
    from prana_b200 import model as pm

    spec, path = _preset_path(args, "stories15m_q8_0")
    model = pm.Model.load(str(path), 0)
    try:
        rng = np.random.default_rng(1234)
        prompt = rng.integers(spec.vocab, size=8).astype(np.uint32)
        steps = spec.ctx - len(prompt)  # 248: the context fills exactly
        stream = torch.cuda.ExternalStream(model.stream())
        pm.generate(model, prompt, steps)  # warm: graphs captured
        torch.cuda.synchronize()
        # e2e: prana_generate (prefill of 7 ids, then the device loop; ids back to the host)
        reps = 5
        e0, e1 = _events(torch)
        e0.record(stream)
        for _ in range(reps):
            got = pm.generate(model, prompt, steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_gen = e0.elapsed_time(e1) / reps
        # value: the device-resident decode loop alone over the same 248 positions
        kv = pm.KvCache(model, spec.ctx)
        pm.prefill(model, kv, prompt[:-1])
        loop = pm.DecodeLoop(model, kv)
        loop.begin(int(prompt[-1]), len(prompt) - 1)
        loop.run(4)
        torch.cuda.synchronize()
        loop.begin(int(prompt[-1]), len(prompt) - 1)
        e0, e1 = _events(torch)
        e0.record(stream)
        loop.run(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_loop = e0.elapsed_time(e1) / steps
        kv.close()
        # CPU oracle: the same generate
        orc.lib().or_pool_set_threads(os.cpu_count() or 1)
        om = orc.OModel(str(path), orc.TIER_AUTO)
        om.generate(prompt, 8)
        t0 = time.perf_counter()
        ref = om.generate(prompt, steps)
        el = time.perf_counter() - t0
        # greedy parity, forced (oracle/parity.py): the prompt's prefill and each of the
        # 248 steps of the GPU's stream, the traced replay reproducing the generated ids
        from oracle.parity import Flips, forced_batch, forced_decode, rel

        okv, gkv = om.kv(spec.ctx), pm.KvCache(model, spec.ctx)
        flips = Flips()
        gated = same = replay = 0
        worst, err = 0.0, None
        try:
            forced_batch(om, okv, model, gkv, prompt[:-1], 0, True, flips, "prompt")
            tok = int(prompt[-1])
            for i in range(len(got)):
                lg_g, lg_o = forced_decode(om, okv, model, gkv, tok, len(prompt) - 1 + i, flips, f"step {i}")
                g = int(np.argmax(lg_g))
                replay += int(g == int(got[i]))
                worst = max(worst, rel(lg_g, lg_o))
                if margin(lg_o) > 1e-3:
                    gated += 1
                    same += int(g == int(np.argmax(lg_o)))
                tok = int(got[i])
        except AssertionError as e:
            err = str(e)
        gkv.close()
        agree = int(np.argmax(np.concatenate([got != ref, [True]])))
        forced = {"steps": len(got), "replay_equals_benchmarked": replay, "margin_gated": gated, "identical": same,
                  "max_logit_rel_err": float(f"{worst:.3g}"), "int8_tie_flips": flips.flips,
                  "f16_kv_tie_flips": flips.kv_flips}
        if err:
            forced["failed"] = err
        wb = spec.weight_bytes_per_token()
        return {
            "metric": "decode tok/s at batch 1 (greedy 248 tokens after an 8-id prompt)", "unit": UNIT,
            "value": round(1000.0 / ms_loop, 1), "ms_per_step": round(ms_loop, 4),
            "e2e": {"value": round(steps * 1000.0 / ms_gen, 1), "unit": UNIT, "path": "prana_generate per call",
                    "h2d_bytes_per_step": round(len(prompt) * 4 / steps, 3), "d2h_bytes_per_step": 4},
            "step_roofline": {"bytes_per_token": wb, "achieved_gbs": round(wb / ms_loop / 1e6, 1),
                              "frac": round(wb / ms_loop / 1e6 / peak, 4),
                              "note": "16 MB per token fits in L2; the step is launch/latency-bound"},
            "cpu_baseline": {"value": round(steps / el, 1), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": f"oracle generate, {steps} tokens, {el:.2f} s"},
            "parity": {"forced": forced, "free_running_identical_prefix": agree},
            "config": {"workload": "stories15m_q8_0", "prompt": len(prompt), "steps": steps, "batch": 1},
        }
    finally:
        model.close()


GEMV_SHAPES = (4096, 11008, 14336)
GEMV_ROWS = (1, 4, 8, 64)


def suite_c2(torch, args, peak):
    """C2: the quantized GEMV/GEMM microbench, K = 4096, weights rotating over
    copies larger than twice L2, activations quantized per row (matmul_*_prefill)."""
    from oracle import oracle as orc
    from prana_b200 import kernels as K
    from prana_b200 import synth
    from prana_b200._ffi import TYPE_NAMES, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

    cols = 4096
    bpw = {TYPE_Q8_0: 34 / 32, TYPE_Q4_0: 18 / 32, TYPE_Q4_K: 144 / 256, TYPE_Q6_K: 210 / 256}
    out = {}
    side = torch.cuda.Stream()
    cpu = {}
    orc.lib().or_pool_set_threads(os.cpu_count() or 1)
    for ty in (TYPE_Q8_0, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K):
        res = {}
        for rows in GEMV_SHAPES:
            raw = synth.matrix(ty, rows, cols, seed=700 + rows)
            wbytes = rows * cols * bpw[ty]
            n_copies = max(4, int(np.ceil(2.2 * 126e6 / wbytes)))
            copies = [K.QuantMatrix(ty, rows, cols, raw) for _ in range(n_copies)]
            fn = K.matmul_q8_prefill if ty == TYPE_Q8_0 else K.matmul_kquant_prefill
            per = {}
            for m in GEMV_ROWS:
                acts = K.quantize_acts(torch.randn(m, cols, device="cuda"))
                iters = 2 * n_copies
                with torch.cuda.stream(side):
                    for w in copies:
                        fn(acts, w)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
                    for i in range(iters):
                        fn(acts, copies[i % n_copies])
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = _events(torch)
                e0.record(side)
                with torch.cuda.stream(side):
                    graph.replay()
                e1.record(side)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1000.0 / iters
                g = cols // 32
                alg = wbytes + m * (cols + 8 * g) + m * rows * 4
                gbs = alg / (us * 1e-6) / 1e9
                per[str(m)] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
                del graph
            res[str(rows)] = per
            if rows == 4096:  # the CPU reference GEMV at batch 1 (the reference's `prana bench` shape family)
                om = orc.OMatrix(ty, rows, cols, raw)
                a = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
                om.matmul(a)
                t0 = time.perf_counter()
                n_it = 0
                while time.perf_counter() - t0 < 1.0:
                    om.matmul(a)
                    n_it += 1
                el = (time.perf_counter() - t0) / n_it
                cpu[TYPE_NAMES[ty]] = {"us": round(el * 1e6, 1), "gbs": round(wbytes / el / 1e9, 2)}
            del copies
        out[TYPE_NAMES[ty]] = res
    return {"metric": "quant GEMV HBM GB/s as % of B200 peak", "unit": "GB/s", "peak": peak, "k": cols,
            "results": out,
            "algorithmic_bytes": "N*K*bpw (GGUF bytes) + M*(K + 8*K/32) + M*N*4",
            "l2": "weights rotate over copies totalling > 2.2 x 126 MB",
            "path": "M <= 8: streaming dp4a GEMV (6-8 rows of Q8_0 / Q4_0 / Q4_K with >= 8192 weight rows: qgemm); "
                    "M > 8: tcgen05 block-scaled int8 GEMM (qgemm); "
                    "consecutive calls chained by programmatic dependent launch, as in the decode step",
            "cpu_baseline": {"results_m1_n4096": cpu, "cores": os.cpu_count(), "kind": "port",
                             "sample": "oracle matmul at batch 1, 1 s per format"},
            "config": {"workload": "gemv_microbench", "k": cols, "n": list(GEMV_SHAPES), "m": list(GEMV_ROWS)}}


def suite_c3(torch, args, peak):
    """C3: Qwen2-0.5B shape, Q4_K/Q6_K-style mixture: prefill 2048 seeded ids,
    then greedy decode 256 over the prefilled cache."""
    from prana_b200 import model as pm

    spec, path = _preset_path(args, "qwen2_0p5b_mix")
    model = pm.Model.load(str(path), 0)
    try:
        c = model.config
        rng = np.random.default_rng(2048)
        prompt = rng.integers(spec.vocab, size=2048).astype(np.uint32)
        steps = 256
        stream = torch.cuda.ExternalStream(model.stream())
        kv = pm.KvCache(model, len(prompt) + steps + 8)
        pm.prefill(model, kv, prompt[:-1])  # warm: the same 2047 rows (buffers sized, kernels loaded)
        torch.cuda.synchronize()
        e0, e1 = _events(torch)
        e0.record(stream)
        pm.prefill(model, kv, prompt[:-1])
        e1.record(stream)
        torch.cuda.synchronize()
        ms_prefill = e0.elapsed_time(e1)
        loop = pm.DecodeLoop(model, kv)
        loop.begin(int(prompt[-1]), len(prompt) - 1)
        loop.run(4)
        torch.cuda.synchronize()
        loop.begin(int(prompt[-1]), len(prompt) - 1)
        e0, e1 = _events(torch)
        e0.record(stream)
        loop.run(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        # e2e: prana_forward per token, host id in and out, continuing the sequence
        toks = loop.tokens(steps)
        pos, tok = len(prompt) - 1 + steps, int(toks[-1])
        n_e2e = 64
        kv2 = pm.KvCache(model, len(prompt) + steps + n_e2e + 8)
        for layer in range(c.n_layers):
            for is_v in (False, True):
                kv2.write(layer, is_v, kv.read(layer, is_v, pos))
        e0, e1 = _events(torch)
        e0.record(stream)
        for _ in range(n_e2e):
            _, tok = pm.forward(model, kv2, tok, pos, want_logits=False)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / n_e2e
        kv2.close()
        kv.close()
        # CPU oracle and greedy parity from seeded KV at 2048 (the oracle's prefill
        # of 2048 tokens alone would take minutes)
        kv_dim = c.kv_dim()
        ctx = 2048
        rows_fn = lambda l, v: seeded_kv_rows(l, v, ctx, kv_dim)  # noqa: E731
        kv3 = pm.KvCache(model, ctx + 64)
        for layer in range(c.n_layers):
            for is_v in (False, True):
                kv3.write(layer, is_v, rows_fn(layer, is_v))
        loop3 = pm.DecodeLoop(model, kv3)
        loop3.begin(17, ctx)
        loop3.run(40)
        follow = loop3.tokens(40)
        kv3.close()
        tps, n_cpu, threads, tier, el, parity = cpu_decode(path, ctx, rows_fn, c.n_layers, kv_dim, 10.0,
                                                           follow=follow)
        parity = {"forced": forced_parity(path, model, ctx, rows_fn, c.n_layers, 17, follow, 16),
                  "free_running": parity}
        kv_bytes = 2 * c.n_layers * (len(prompt) + steps // 2) * kv_dim * 2
        bt = spec.weight_bytes_per_token() + kv_bytes
        return {
            "metric": "decode tok/s at batch 1 (after a 2048-token prefill)", "unit": UNIT,
            "value": round(1000.0 / ms, 1), "ms_per_step": round(ms, 4),
            "e2e": {"value": round(1000.0 / ms_e2e, 1), "unit": UNIT, "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 8},
            "prefill": {"tokens": len(prompt) - 1, "ms": round(ms_prefill, 2),
                        "tok_s": round((len(prompt) - 1) * 1000.0 / ms_prefill, 1),
                        "path": "tensor-core GEMMs over the prompt rows; f32 in-window attention"},
            "step_roofline": {"bytes_per_token": bt, "achieved_gbs": round(bt / ms / 1e6, 1),
                              "frac": round(bt / ms / 1e6 / peak, 4)},
            "cpu_baseline": {"value": round(tps, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{n_cpu} greedy tokens at ctx {ctx + 1}.. from seeded KV, {tier} tier, "
                                       f"{el:.1f} s"},
            "parity": parity,
            "config": {"workload": "qwen2_0p5b_mix", "prefill": len(prompt), "steps": steps, "batch": 1,
                       "types": "Q4_0 (attn q/k/o, ffn gate/up, embedding), Q8_0 (attn v, output), Q6_K (ffn down)"},
        }
    finally:
        model.close()


def suite_c4q8(torch, args, peak):
    """C4, Q8_0 variant: the 8B shape in Q8_0 at ctx 4096, batch 1."""
    from prana_b200 import model as pm

    spec, path = _preset_path(args, "llama3_8b_q8_0")
    model = pm.Model.load(str(path), 0)
    try:
        c = model.config
        kv_dim = c.kv_dim()
        steps, warm = 64, 8
        kv = pm.KvCache(model, args.ctx + steps + warm + 80)
        rows_fn = lambda l, v: seeded_kv_rows(l, v, args.ctx, kv_dim)  # noqa: E731
        for layer in range(c.n_layers):
            for is_v in (False, True):
                kv.write(layer, is_v, rows_fn(layer, is_v))
        stream = torch.cuda.ExternalStream(model.stream())
        loop = pm.DecodeLoop(model, kv)
        loop.begin(17, args.ctx)
        loop.run(warm)
        torch.cuda.synchronize()
        e0, e1 = _events(torch)
        e0.record(stream)
        loop.run(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        toks = loop.tokens(warm + steps)
        pos, tok = args.ctx + warm + steps, int(toks[-1])
        e0, e1 = _events(torch)
        e0.record(stream)
        for _ in range(32):
            _, tok = pm.forward(model, kv, tok, pos, want_logits=False)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / 32
        kv.close()
        tps, n_cpu, threads, tier, el, parity = cpu_decode(path, args.ctx, rows_fn, c.n_layers, kv_dim, 12.0,
                                                           follow=toks)
        parity = {"forced": forced_parity(path, model, args.ctx, rows_fn, c.n_layers, 17, toks, 4),
                  "free_running": parity}
        bt = spec.weight_bytes_per_token() + 2 * c.n_layers * (args.ctx + warm + steps // 2) * kv_dim * 2
        return {
            "metric": METRIC, "unit": UNIT, "value": round(1000.0 / ms, 2), "ms_per_step": round(ms, 4),
            "e2e": {"value": round(1000.0 / ms_e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 8},
            "step_roofline": {"bytes_per_token": bt, "achieved_gbs": round(bt / ms / 1e6, 1),
                              "frac": round(bt / ms / 1e6 / peak, 4)},
            "cpu_baseline": {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{n_cpu} greedy tokens at ctx {args.ctx + 1}.. from the same seeded KV, fed "
                                       f"the GPU's tokens, {tier} tier, {el:.1f} s"},
            "parity": parity,
            "config": {"workload": "llama3_8b_q8_0", "ctx": args.ctx, "batch": 1},
        }
    finally:
        model.close()


def suite_c5(torch, args, peak):
    """C5: greedy speculative decode, Qwen2-0.5B-shape Q8_0 draft and 1.5B-shape
    Q8_0 target over a shared vocabulary (151936), k = 4, context 1024; the
    pair's shared-code construction (synth.py C5_*) makes ~60 % of the drafted
    tokens acceptable.  Plain greedy decode of the target is timed beside it."""
    from oracle import oracle as orc
    from prana_b200 import model as pm

    _, dpath = _preset_path(args, "qwen2_0p5b_q8_0_spec")
    tspec, tpath = _preset_path(args, "qwen2_1p5b_q8_0_spec")
    dm, tm = pm.Model.load(str(dpath), 0), pm.Model.load(str(tpath), 0)
    try:
        rng = np.random.default_rng(16)
        prompt = rng.integers(tspec.vocab, size=16).astype(np.uint32)
        steps, k = 256, 4
        stream = torch.cuda.ExternalStream(tm.stream())
        # warm at the timed size: the first allocations of this cache capacity and
        # of the prompt's prefill buffers happen outside the timed calls
        pm.generate(tm, prompt, steps)
        pm.generate_speculative(tm, dm, prompt, steps, k)
        torch.cuda.synchronize()
        e0, e1 = _events(torch)
        e0.record(stream)
        plain = pm.generate(tm, prompt, steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_plain = e0.elapsed_time(e1)
        e0, e1 = _events(torch)
        e0.record(stream)
        spec, (proposed, accepted) = pm.generate_speculative(tm, dm, prompt, steps, k)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_spec = e0.elapsed_time(e1)
        # CPU oracle: the reference's own loops over the same pair, bounded samples
        orc.lib().or_pool_set_threads(os.cpu_count() or 1)
        od, ot = orc.OModel(str(dpath), orc.TIER_AUTO), orc.OModel(str(tpath), orc.TIER_AUTO)
        n_cpu = 12
        t0 = time.perf_counter()
        cpu_plain = ot.generate(prompt, n_cpu)
        el_plain = time.perf_counter() - t0
        t0 = time.perf_counter()
        cpu_spec, (cp, ca) = ot.generate_speculative(od, prompt, n_cpu, k)
        el_spec = time.perf_counter() - t0
        return {
            "metric": "speculative decode tok/s at batch 1 (greedy, k = 4)", "unit": UNIT,
            "value": round(len(spec) * 1000.0 / ms_spec, 1),
            "plain_greedy": {"value": round(len(plain) * 1000.0 / ms_plain, 1), "unit": UNIT,
                             "path": "prana_generate: prefill, then the device decode loop"},
            "e2e": {"value": round(len(spec) * 1000.0 / ms_spec, 1), "unit": UNIT,
                    "path": "prana_generate_speculative per call (draft steps and the (k+1)-row verify host-driven)",
                    "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
            "acceptance": round(accepted / max(proposed, 1), 3), "proposed": proposed, "accepted": accepted,
            "speedup_vs_plain": round(ms_plain / ms_spec * len(spec) / max(len(plain), 1), 3),
            "cpu_baseline": {"value": round(n_cpu / el_spec, 3), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "plain_value": round(n_cpu / el_plain, 3), "acceptance": round(ca / max(cp, 1), 3),
                             "sample": f"oracle generate_speculative and generate, {n_cpu} tokens each, "
                                       f"{el_spec:.1f} s and {el_plain:.1f} s"},
            "parity": {"spec_equals_greedy": bool(np.array_equal(spec, plain)),
                       "cpu_spec_equals_cpu_greedy": bool(np.array_equal(cpu_spec, cpu_plain)),
                       "gpu_greedy_prefix_equals_cpu": int(np.argmax(np.concatenate([plain[:n_cpu] != cpu_plain,
                                                                                     [True]])))},
            "config": {"workload": "qwen2_0p5b_q8_0 draft -> qwen2_1p5b_q8_0 target", "k": k, "prompt": len(prompt),
                       "steps": steps, "ctx": tspec.ctx, "batch": 1},
        }
    finally:
        dm.close()
        tm.close()


SUITE = {"c1": suite_c1, "c2": suite_c2, "c3": suite_c3, "c4q8": suite_c4q8, "c5": suite_c5}


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
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
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
    cap = args.ctx + 3 * (args.warmup + args.steps) + 16
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
    if dist:
        # align the ranks on the device: one more (untimed) step, whose exchanges
        # finish together on every rank, precedes the start event in stream order
        loop.run(1)
    e0.record(stream)
    loop.run(args.steps)
    e1.record(stream)
    barrier()
    clk = clocks.stop(t_region, time.monotonic())
    ms = e0.elapsed_time(e1) / args.steps
    n_loop = args.warmup + args.steps + (1 if dist else 0)
    toks = loop.tokens(n_loop)
    # ---- e2e: C-ABI call per token with host buffers
    pos = args.ctx + n_loop
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
    # ---- the device loop with temperature sampling (Sampler::sample on the device)
    sampled = None
    if world == 1:
        from prana_b200.sampler import Sampler

        loop.begin(int(tok), pos, sampler=Sampler(SAMPLE_TEMP, SAMPLE_SEED))
        loop.run(args.warmup)
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        loop.run(args.steps)
        g1.record(stream)
        barrier()
        ms_s = g0.elapsed_time(g1) / args.steps
        pos += args.warmup + args.steps
        sampled = {"value": round(1000.0 / ms_s, 3), "unit": UNIT, "ms_per_step": round(ms_s, 4),
                   "temperature": SAMPLE_TEMP, "seed": SAMPLE_SEED,
                   "path": "device decode loop, Sampler::sample on the device (logits stay in HBM)"}
    batch = batch_decode(torch, model, args, stream) if world == 1 and args.batch_seqs > 0 else None
    roof = gemv_roofline(torch, peak) if rank == 0 else None
    cpu = cpu8 = parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows_fn = lambda l, v: seeded_kv_rows(l, v, args.ctx, kv_dim)  # noqa: E731
        tps, steps, threads, tier, el, parity = cpu_decode(path, args.ctx, rows_fn, c.n_layers, kv_dim,
                                                           args.cpu_seconds, follow=toks)
        cpu = {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{steps} greedy tokens at ctx {args.ctx + 1}.. from the same seeded KV, fed the GPU's "
                         f"tokens, {tier} tier, {el:.1f} s"}
        # the reference's default worker count, min(cores, 8) (threading.rs:46-53)
        t8 = min(os.cpu_count() or 1, 8)
        tps8, steps8, _, tier8, el8, _ = cpu_decode(path, args.ctx, rows_fn, c.n_layers, kv_dim,
                                                    args.cpu_seconds / 2, threads=t8)
        cpu8 = {"value": round(tps8, 4), "unit": UNIT, "cores": t8, "kind": "port",
                "sample": f"{steps8} greedy tokens at ctx {args.ctx + 1}.., {tier8} tier, {el8:.1f} s"}
        parity = {"forced": forced_parity(path, model, args.ctx, rows_fn, c.n_layers, 17, toks, 6),
                  "free_running": parity}
    suite = {}
    if rank == 0 and world == 1:
        todo = args.configs.split(",") if args.configs is not None else ["c1", "c2", "c3", "c4q8", "c5"]
        for name in [x.strip() for x in todo if x.strip()]:
            fn = SUITE.get(name)
            if fn is None:
                suite[name] = {"error": "unknown config"}
                continue
            try:
                suite[name] = fn(torch, args, peak)
            except Exception as e:  # one config's failure is reported, not fatal to the line
                suite[name] = {"error": f"{type(e).__name__}: {e}"}
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
                    "d2h_bytes_per_step": 8},
            "roofline": roof, "peak_kind": peak_kind,
            "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": round(step_gbs, 1),
                              "frac": round(step_gbs / peak, 4)},
            "cpu_baseline": cpu, "cpu_baseline_default_threads": cpu8, "parity": parity,
            "sampled_decode": sampled, "batch_decode": batch, "clocks": clk,
            "gpu_launches": launches_per_step(spec, world, model.peer_exchange) * args.steps,
            "load_s": round(t_load, 1),
            "configs": suite or None,
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
