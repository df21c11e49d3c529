"""Multi-sequence decode (prana_forward_multi) against per-sequence decode.

Twelve independent sequences, each with its own KV cache holding a different
seeded history, advance one token each in one pass (GEMV rows in chunks of 8,
attention per sequence).  The reference has no such batch: its equivalent is
one forward (infer.rs:142-211) per sequence, which is what each row is checked
against here, through the single-sequence GPU path that the oracle tests pin.
Rows differ from it only by f32 summation order (batch-8 vs batch-1 GEMV), so
logits must agree within TOL and the greedy token wherever the top-2 margin
exceeds TOL; two consecutive multi steps are checked, so the K/V rows the first
one wrote are exercised by the second.
"""
import numpy as np
import pytest

from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q6_K, TYPE_Q8_0, PranaError

pytestmark = pytest.mark.gpu

TOL = 2e-2
N_SEQ = 12

SPECS = {
    "llama_q8": synth.ModelSpec("llama", 256, 512, 3, 8, 4, 32, 1000, 128, 10000.0, 1e-5, seed=31),
    "llama_q4_0_hd64": synth.ModelSpec("llama", 256, 768, 2, 4, 2, 64, 777, 96, 5e5, 1e-5, seed=32).with_types(TYPE_Q4_0),
    "qwen2_mix": synth.ModelSpec("qwen2", 224, 512, 2, 7, 1, 32, 1200, 128, 1e6, 1e-6, has_bias=True, seed=33,
                                 type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                                 type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                                 type_output=TYPE_Q8_0),
}


def rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(float(np.max(np.abs(b))), 1e-30))


def margin(lg):
    s = np.sort(lg)
    return float((s[-1] - s[-2]) / max(float(np.max(np.abs(lg))), 1e-30))


def histories(vocab, seed=7):
    rng = np.random.default_rng(seed)
    return [rng.integers(vocab, size=1 + (i * 5) % 11) for i in range(N_SEQ)]


def fill(model, hist):
    caches = []
    for h in hist:
        kv = pm.KvCache(model, 32)
        for pos, t in enumerate(h):
            pm.forward(model, kv, int(t), pos, want_logits=False)
        caches.append(kv)
    return caches


@pytest.mark.parametrize("name", list(SPECS))
def test_forward_multi_matches_per_sequence(tmp_path, gpu, name):
    path = tmp_path / f"{name}.gguf"
    synth.write_gguf(SPECS[name], path)
    m = pm.Model.load(str(path), 0)
    try:
        vocab = m.config.vocab_size
        hist = histories(vocab)
        multi, single = fill(m, hist), fill(m, hist)
        rng = np.random.default_rng(11)
        pos = np.array([len(h) for h in hist], dtype=np.uint64)
        gated = agree = 0
        worst = 0.0
        for step in range(2):
            toks = rng.integers(vocab, size=N_SEQ)
            lg, am = pm.forward_multi(m, multi, toks, pos + step)
            assert lg.shape == (N_SEQ, vocab) and am.shape == (N_SEQ,)
            for i in range(N_SEQ):
                lr, tr = pm.forward(m, single[i], int(toks[i]), int(pos[i]) + step)
                worst = max(worst, rel(lg[i], lr))
                assert int(am[i]) == int(np.argmax(lg[i]))
                if margin(lr) > TOL:
                    gated += 1
                    agree += int(am[i] == tr)
        assert worst < TOL, worst
        assert agree == gated
        # the last step's K/V rows of every sequence (layer 0, the newest position)
        for i in range(N_SEQ):
            rows = int(pos[i]) + 2
            for is_v in (False, True):
                a = multi[i].read(0, is_v, rows).view(np.float16).astype(np.float32)
                b = single[i].read(0, is_v, rows).view(np.float16).astype(np.float32)
                assert np.max(np.abs(a - b)) <= 2e-3 * max(1.0, float(np.max(np.abs(b))))
        for kv in multi + single:
            kv.close()
    finally:
        m.close()


def test_forward_multi_rejects_shared_cache(tmp_path, gpu):
    path = tmp_path / "m.gguf"
    synth.write_gguf(SPECS["llama_q8"], path)
    m = pm.Model.load(str(path), 0)
    try:
        kv = pm.KvCache(m, 16)
        with pytest.raises(PranaError, match="share a cache"):
            pm.forward_multi(m, [kv, kv], [1, 2], [0, 0])
        kv.close()
    finally:
        m.close()
