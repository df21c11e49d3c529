"""Model-level GPU parity against the CPU oracle on seeded GGUF models.

Every comparison runs the oracle in forced mode (tests/parity.py): at each
quantization site both sides' int8 rows must be equal or differ by one step at
a rounding tie of the oracle's own value, and the oracle then continues with
the GPU's rows.  Logits of every step must match within 1e-3 max relative
error and the greedy token must be identical wherever the oracle's top-2
margin exceeds 1e-3 -- for single-token decode, prefill, forward_batch
(speculative verify), greedy generation and the device decode loop.
"""
import numpy as np
import pytest

from oracle.parity import Flips, check_logits, forced_batch, forced_decode
from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu

SPECS = {
    "llama_q8": synth.ModelSpec("llama", 256, 512, 3, 8, 4, 32, 1000, 128, 10000.0, 1e-5, seed=1),
    "llama_q4_0": synth.ModelSpec("llama", 256, 768, 2, 4, 4, 64, 777, 96, 5e5, 1e-5, seed=2).with_types(TYPE_Q4_0),
    "llama_kq": synth.ModelSpec("llama", 512, 768, 2, 4, 1, 128, 900, 96, 5e5, 1e-5, seed=3,
                                type_embd=TYPE_Q4_K, type_q=TYPE_Q4_K, type_k=TYPE_Q6_K, type_v=TYPE_Q6_K,
                                type_o=TYPE_Q4_K, type_gate=TYPE_Q4_K, type_up=TYPE_Q4_K, type_down=TYPE_Q6_K,
                                type_output=TYPE_Q6_K),
    "qwen2_mix": synth.ModelSpec("qwen2", 224, 512, 3, 7, 1, 32, 1200, 128, 1e6, 1e-6, has_bias=True, seed=4,
                                 type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                                 type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                                 type_output=TYPE_Q8_0),
    # a second qwen2-shaped model over the same vocabulary: the cross draft
    "qwen2_draft": synth.ModelSpec("qwen2", 128, 256, 2, 4, 2, 32, 1200, 128, 1e6, 1e-6, has_bias=True,
                                   seed=44).with_types(TYPE_Q8_0),
    "stories_shape": synth.STORIES15M_Q8,
}


@pytest.fixture(scope="module")
def models(tmp_path_factory, gpu, oracle):
    d = tmp_path_factory.mktemp("models")
    out = {}
    for name, spec in SPECS.items():
        path = d / f"{name}.gguf"
        synth.write_gguf(spec, path)
        out[name] = (path, oracle.OModel(str(path), oracle.TIER_SCALAR), pm.Model.load(str(path), 0))
    yield out
    for _, _, gm in out.values():
        gm.close()


def copy_cache(okv, gkv, n_layers, rows):
    for layer in range(n_layers):
        for is_v in (False, True):
            gkv.write(layer, is_v, okv.layer(layer, is_v)[:rows])


ALL = [n for n in SPECS if n != "qwen2_draft"]


@pytest.mark.parametrize("name", ALL)
def test_forward_teacher_forced(models, name):
    """Each decode step runs on both sides from the same KV cache (the oracle's);
    the oracle is forced with the GPU's int8 rows after every difference is proven
    a rounding tie; logits within 1e-3 and the greedy token on every step."""
    _, om, gm = models[name]
    c = gm.config
    steps = 16
    okv, gkv = om.kv(steps + 1), pm.KvCache(gm, steps + 1)
    rng = np.random.default_rng(5)
    flips, gated = Flips(), 0
    for pos in range(steps):
        copy_cache(okv, gkv, c.n_layers, pos)
        tok = int(rng.integers(c.vocab_size))
        lg_g, lg_o = forced_decode(om, okv, gm, gkv, tok, pos, flips, f"{name} pos {pos}")
        gated += check_logits(lg_g, lg_o, f"{name} pos {pos}")
        # the forward path without the trace gives the same logits
        lg_p, nxt = pm.forward(gm, gkv, tok, pos)
        assert np.array_equal(lg_p, lg_g) and nxt == int(np.argmax(lg_g))
    assert flips.bounded(), f"{name}: {flips.flips} flipped activations of {flips.total}"
    assert gated >= steps // 2


@pytest.mark.parametrize("name", ["llama_q8", "qwen2_mix", "llama_kq", "llama_q4_0"])
def test_prefill_then_decode(models, name):
    """prefill (f32 in-window attention) site by site, the K/V rows it writes, and
    the first decode step over the prefilled cache."""
    _, om, gm = models[name]
    c = gm.config
    rng = np.random.default_rng(6)
    toks = rng.integers(c.vocab_size, size=21).astype(np.uint32)
    n = len(toks)
    okv, gkv = om.kv(40), pm.KvCache(gm, 40)
    flips = Flips()
    forced_batch(om, okv, gm, gkv, toks, 0, True, flips, f"{name} prefill")
    lg_g, lg_o = forced_decode(om, okv, gm, gkv, 9, n, flips, f"{name} decode after prefill")
    check_logits(lg_g, lg_o, f"{name} decode after prefill")
    assert flips.bounded()
    # the prefill entry point computes the traced pass's cache rows
    kv2 = pm.KvCache(gm, 40)
    pm.prefill(gm, kv2, toks)
    for layer in range(c.n_layers):
        for is_v in (False, True):
            assert np.array_equal(kv2.read(layer, is_v, n), gkv.read(layer, is_v, n))


@pytest.mark.parametrize("name", ["llama_q8", "qwen2_mix", "llama_kq"])
@pytest.mark.parametrize("n", [1, 5, 8, 11])
def test_forward_batch(models, name, n):
    """forward_batch (the speculative verify pass) row by row at 1e-3."""
    _, om, gm = models[name]
    c = gm.config
    rng = np.random.default_rng(7)
    pre = rng.integers(c.vocab_size, size=6).astype(np.uint32)
    toks = rng.integers(c.vocab_size, size=n).astype(np.uint32)
    okv, gkv = om.kv(40), pm.KvCache(gm, 40)
    om.prefill(okv, pre)
    copy_cache(okv, gkv, c.n_layers, len(pre))
    flips = Flips()
    lg_g, lg_o = forced_batch(om, okv, gm, gkv, toks, len(pre), False, flips, f"{name} n={n}")
    for i in range(n):
        check_logits(lg_g[i], lg_o[i], f"{name} n={n} row {i}")
    assert flips.bounded()
    # the untraced entry point gives the same rows and their argmax
    kv2 = pm.KvCache(gm, 40)
    copy_cache(okv, kv2, c.n_layers, len(pre))
    lg_p, am = pm.forward_batch(gm, kv2, toks, len(pre))
    assert np.array_equal(lg_p, lg_g)
    assert np.array_equal(am, np.argmax(lg_p, axis=1))


@pytest.mark.parametrize("name", ALL)
def test_generate_greedy_tokens(models, name):
    """generate (prefill, then the device decode loop) against the oracle: the GPU's
    tokens are replayed step by step through the traced path (which must give the
    same ids), and each step is checked against the forced oracle; every token
    whose oracle top-2 margin exceeds 1e-3 must be the oracle's argmax."""
    _, om, gm = models[name]
    c = gm.config
    rng = np.random.default_rng(8)
    prompt = rng.integers(c.vocab_size, size=8).astype(np.uint32)
    steps = 40
    got = pm.generate(gm, prompt, steps)
    assert len(got) == min(steps, c.seq_len - len(prompt))
    p = len(prompt)
    okv, gkv = om.kv(p + steps), pm.KvCache(gm, p + steps)
    flips = Flips()
    forced_batch(om, okv, gm, gkv, prompt[:-1], 0, True, flips, f"{name} prompt")
    tok, gated = int(prompt[-1]), 0
    for i in range(len(got)):
        pos = p - 1 + i
        lg_g, lg_o = forced_decode(om, okv, gm, gkv, tok, pos, flips, f"{name} step {i}")
        assert int(np.argmax(lg_g)) == int(got[i]), f"{name}: step {i} of the decode loop differs from the traced pass"
        gated += check_logits(lg_g, lg_o, f"{name} step {i}")
        tok = int(got[i])
    assert flips.bounded()
    assert gated >= len(got) // 2


@pytest.mark.parametrize("draft", ["qwen2_mix", "qwen2_draft"])
def test_generate_speculative_equals_greedy(models, draft):
    """generate_speculative emits exactly the target's greedy sequence, with the
    target as its own draft and with a different draft model (gguf.rs:745-846)."""
    _, om_t, target = models["qwen2_mix"]
    _, om_d, dm = models[draft]
    rng = np.random.default_rng(9)
    prompt = rng.integers(target.config.vocab_size, size=6).astype(np.uint32)
    plain = pm.generate(target, prompt, 30)
    spec, (proposed, accepted) = pm.generate_speculative(target, dm, prompt, 30, 4)
    assert np.array_equal(spec, plain)
    assert proposed >= accepted
    if draft == "qwen2_mix":
        assert accepted > 0
    # the oracle's speculative loop over the same pair proposes and accepts the same way
    # wherever its own greedy run agrees with the GPU's
    ref, _ = om_t.generate_speculative(om_d, prompt, 30, 4)
    assert np.array_equal(ref, om_t.generate(prompt, 30))


def test_decode_loop_matches_generate(models):
    _, _, gm = models["llama_q8"]
    prompt = np.array([3, 14, 15, 92, 65], np.uint32)
    ref = pm.generate(gm, prompt, 20)
    kv = pm.KvCache(gm, 64)
    pm.prefill(gm, kv, prompt[:-1])
    loop = pm.DecodeLoop(gm, kv)
    loop.begin(int(prompt[-1]), len(prompt) - 1)
    loop.run(10)
    loop.run(10)
    assert np.array_equal(loop.tokens(64)[:20], ref[:20])
