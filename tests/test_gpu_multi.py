"""Multi-sequence decode (prana_forward_multi) against the CPU oracle.

Twelve independent sequences, each with its own KV cache holding a different
seeded history, advance one token each in one pass (GEMV rows in chunks of 8,
one attention launch over all sequences).  The reference has no such batch:
its equivalent is one forward (infer.rs:142-211) per sequence, which is what
each row is checked against -- the oracle's forward, forced with that row's
int8 activations after every difference is proven a rounding tie
(tests/parity.py) -- at 1e-3 on the logits and on the greedy token wherever
the top-2 margin exceeds 1e-3.  Two consecutive multi steps are checked, so the
K/V rows the first one wrote are exercised by the second.
"""
import numpy as np
import pytest

from oracle.parity import Flips, check_logits, check_trace, gpu_kv_rows, row_trace
from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q6_K, TYPE_Q8_0, PranaError

pytestmark = pytest.mark.gpu

N_SEQ = 12

SPECS = {
    "llama_q8": synth.ModelSpec("llama", 256, 512, 3, 8, 4, 32, 1000, 128, 10000.0, 1e-5, seed=31),
    "llama_q4_0_hd64": synth.ModelSpec("llama", 256, 768, 2, 4, 2, 64, 777, 96, 5e5, 1e-5, seed=32).with_types(TYPE_Q4_0),
    "qwen2_mix": synth.ModelSpec("qwen2", 224, 512, 2, 7, 1, 32, 1200, 128, 1e6, 1e-6, has_bias=True, seed=33,
                                 type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                                 type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                                 type_output=TYPE_Q8_0),
}


def histories(vocab, seed=7):
    rng = np.random.default_rng(seed)
    return [rng.integers(vocab, size=1 + (i * 5) % 11) for i in range(N_SEQ)]


@pytest.mark.parametrize("name", list(SPECS))
def test_forward_multi_matches_oracle(tmp_path, gpu, oracle, name):
    path = tmp_path / f"{name}.gguf"
    synth.write_gguf(SPECS[name], path)
    om = oracle.OModel(str(path), oracle.TIER_SCALAR)
    m = pm.Model.load(str(path), 0)
    try:
        c = m.config
        hist = histories(c.vocab_size)
        okvs, gkvs = [], []
        for h in hist:  # each history through the oracle, its cache copied to the GPU
            okv = om.kv(32)
            for pos, t in enumerate(h):
                om.forward(okv, int(t), pos, want_logits=False)
            gkv = pm.KvCache(m, 32)
            for layer in range(c.n_layers):
                for is_v in (False, True):
                    gkv.write(layer, is_v, okv.layer(layer, is_v)[:len(h)])
            okvs.append(okv)
            gkvs.append(gkv)
        rng = np.random.default_rng(11)
        pos = np.array([len(h) for h in hist], dtype=np.uint64)
        flips, gated = Flips(), 0
        for step in range(2):
            toks = rng.integers(c.vocab_size, size=N_SEQ)
            lg, q, s = pm.forward_multi_trace(m, gkvs, toks, pos + step)
            for i in range(N_SEQ):
                qi, si = row_trace(q, s, c, N_SEQ, i)
                p_i = int(pos[i]) + step
                kv_g = gpu_kv_rows(gkvs[i], c.n_layers, p_i, 1)
                lo, q_o, s_o, v_o, kv_o, kv_v = om.forward_trace(okvs[i], int(toks[i]), p_i, with_values=True,
                                                                  force=(qi, si), force_kv=kv_g)
                flips.check_kv(kv_g, kv_o, kv_v, f"{name} step {step} seq {i}", c.n_kv_heads * c.head_dim)
                check_trace(c, qi, si, q_o, s_o, v_o, flips, f"{name} step {step} seq {i}")
                gated += check_logits(lg[i], lo, f"{name} step {step} seq {i}")
        assert flips.bounded()
        assert gated >= N_SEQ
        for kv in gkvs:
            kv.close()
    finally:
        m.close()


def test_forward_multi_entry_point_equals_traced_pass(tmp_path, gpu):
    """The untraced entry point computes the traced pass's rows and their argmax."""
    path = tmp_path / "m.gguf"
    synth.write_gguf(SPECS["qwen2_mix"], path)
    m = pm.Model.load(str(path), 0)
    try:
        vocab = m.config.vocab_size
        hist = histories(vocab)
        a_kv, b_kv = [], []
        for h in hist:
            for lst in (a_kv, b_kv):
                kv = pm.KvCache(m, 32)
                for p, t in enumerate(h):
                    pm.forward(m, kv, int(t), p, want_logits=False)
                lst.append(kv)
        pos = [len(h) for h in hist]
        toks = np.arange(N_SEQ) * 37 % vocab
        lg_t, _, _ = pm.forward_multi_trace(m, a_kv, toks, pos)
        lg, am = pm.forward_multi(m, b_kv, toks, pos)
        assert np.array_equal(lg, lg_t)
        assert np.array_equal(am, np.argmax(lg, axis=1))
        for kv in a_kv + b_kv:
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
