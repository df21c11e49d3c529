"""Tensor-parallel parity worker, launched by tests/test_gpu_tp.py under
torch.distributed.run (one process per GPU).

Every rank loads its shard of a seeded GGUF model; rank 0 also loads the whole
model on its GPU.  Both decode the same teacher-forced token sequence from
their own KV caches; the sharded logits must match the single-GPU logits
within TOL (the ranks' partial products are summed in a different order, so
an activation can round the other way at a tie) and the greedy token must
agree wherever the top-2 margin exceeds TOL.  The graph-driven decode loop of
the sharded model must reproduce its own step-by-step tokens exactly.
"""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from prana_b200 import model as pm  # noqa: E402
from prana_b200 import synth  # noqa: E402
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q6_K, TYPE_Q8_0  # noqa: E402

TOL = 2e-2
SPECS = {
    "llama_q8": synth.ModelSpec("llama", 256, 768, 2, 8, 4, 32, 1000, 128, 10000.0, 1e-5, seed=21),
    "qwen2_mix": synth.ModelSpec("qwen2", 256, 512, 2, 8, 2, 32, 1200, 128, 1e6, 1e-6, has_bias=True, seed=22,
                                 type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                                 type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                                 type_output=TYPE_Q8_0),
}


def rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(float(np.max(np.abs(b))), 1e-30))


def margin(lg):
    s = np.sort(lg)
    return float((s[-1] - s[-2]) / max(float(np.max(np.abs(lg))), 1e-30))


def main():
    name, path = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))  # host side only: the id and barriers
    spec = SPECS[name]
    obj = [None]
    if rank == 0:
        synth.write_gguf(spec, path)
        obj[0] = pm.tp_unique_id()
    dist.broadcast_object_list(obj, src=0)
    tp = pm.Model.load(path, local, tp=(world, rank, obj[0]))
    ref = pm.Model.load(path, local) if rank == 0 else None
    c = tp.config
    steps = 20
    toks = np.random.default_rng(3).integers(c.vocab_size, size=steps)
    kv = pm.KvCache(tp, steps + 8)
    kv_ref = pm.KvCache(ref, steps + 8) if ref else None
    worst, gated, agree, step_toks = 0.0, 0, 0, []
    for pos, t in enumerate(toks):
        lg, tok = pm.forward(tp, kv, int(t), pos)
        step_toks.append(int(tok))
        if ref:
            lr, tr = pm.forward(ref, kv_ref, int(t), pos)
            worst = max(worst, rel(lg, lr))
            if margin(lr) > TOL:
                gated += 1
                agree += int(tok == tr)
    # prefill (more rows than the peer exchange holds: the NCCL path) then a
    # 4-row verify batch (the peer path) against the single-GPU model
    kvb = pm.KvCache(tp, steps + 8)
    pm.prefill(tp, kvb, toks[:12])
    lgb, amb = pm.forward_batch(tp, kvb, toks[12:16], 12)
    if ref:
        kvb_ref = pm.KvCache(ref, steps + 8)
        pm.prefill(ref, kvb_ref, toks[:12])
        lrb, arb = pm.forward_batch(ref, kvb_ref, toks[12:16], 12)
        kvb_ref.close()
        for i in range(4):
            worst = max(worst, rel(lgb[i], lrb[i]))
            if margin(lrb[i]) > TOL:
                gated += 1
                agree += int(amb[i] == arb[i])
    kvb.close()
    # graph-driven decode loop on the sharded model, from a fresh cache: greedy
    # from toks[0]; its tokens must equal the step-by-step greedy chain
    kv2 = pm.KvCache(tp, steps + 8)
    loop = pm.DecodeLoop(tp, kv2)
    loop.begin(int(toks[0]), 0)
    loop.run(8)
    got = [int(x) for x in loop.tokens(8)]
    kv3 = pm.KvCache(tp, steps + 8)
    chain, t = [], int(toks[0])
    for pos in range(8):
        _, t = pm.forward(tp, kv3, t, pos, want_logits=False)
        chain.append(int(t))
    ok_loop = got == chain
    res = {"rank": rank, "worst_rel": worst, "gated": gated, "agree": agree, "loop_equal": ok_loop}
    for m in (kv, kv2, kv3):
        m.close()
    if kv_ref:
        kv_ref.close()
    tp.close()
    if ref:
        ref.close()
    dist.barrier()
    dist.destroy_process_group()
    print(json.dumps(res), flush=True)
    if rank == 0 and not (worst < TOL and agree == gated):
        sys.exit(1)
    if not ok_loop:
        sys.exit(2)


if __name__ == "__main__":
    main()
