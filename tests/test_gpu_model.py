"""Model-level GPU parity against the CPU oracle on seeded GGUF models.

Logits must match within 1e-3 normwise relative error (max|gpu - oracle| /
max|oracle|, the BASELINE logits tolerance); greedy tokens must be identical
wherever the oracle's top-2 margin exceeds that tolerance.
"""
import numpy as np
import pytest

from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
# Free-running multi-step comparisons inherit any earlier +-1 activation rounding
# flip through the KV cache; the reference's own scalar and AVX2/VNNI tiers differ
# by up to 1.3e-2 on these models for that reason (measured), so those tests use
# this bound while the per-step BASELINE tolerance is enforced by the
# teacher-forced, flip-aware test.
FREE_TOL = 2e-2


def rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(float(np.max(np.abs(b))), 1e-30))


def margin(lg):
    s = np.sort(lg)
    return float((s[-1] - s[-2]) / max(float(np.max(np.abs(lg))), 1e-30))


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


def trace_sites(c):
    """(offset, length) of every traced activation row, in forward order."""
    sites, off = [], 0
    for _ in range(c.n_layers):
        for n in (c.dim, c.n_heads * c.head_dim, c.dim, c.hidden_dim):
            sites.append((off, n))
            off += n
    sites.append((off, c.dim))
    return sites


@pytest.mark.parametrize("name", list(SPECS))
def test_forward_teacher_forced_flip_aware(models, name):
    """Each decode step is run on both sides from the same (oracle) KV cache and
    every int8 activation row both sides quantize is compared.

    * Up to the first row where the two sides' int8 activations differ, they are
      identical; at that row every difference is a single +-1 rounding flip of an
      element that sat on a rounding boundary (1-ulp f32 differences upstream).
    * Steps with no flip must give logits within LOGIT_TOL and the same greedy
      token whenever the top-2 margin exceeds LOGIT_TOL.
    * Flips are rare (they are what makes the reference's own scalar and SIMD
      tiers diverge by up to ~1e-2 on these models).
    """
    _, om, gm = models[name]
    c = gm.config
    sites = trace_sites(c)
    steps = 16
    okv, gkv = om.kv(steps + 1), pm.KvCache(gm, steps + 1)
    rng = np.random.default_rng(5)
    flips = total = flip_steps = 0
    for pos in range(steps):
        for layer in range(c.n_layers):
            for is_v in (False, True):
                gkv.write(layer, is_v, okv.layer(layer, is_v)[:pos])
        tok = int(rng.integers(c.vocab_size))
        lg_o, q_o, s_o, v_o = om.forward_trace(okv, tok, pos, with_values=True)
        lg_g, q_g, s_g = pm.forward_trace(gm, gkv, tok, pos)
        first = None
        for off, n in sites:
            if first is not None:
                break  # downstream of a flip the inputs legitimately differ
            d = q_g[off:off + n].astype(np.int32) - q_o[off:off + n]
            so, sg = s_o[off // 32:(off + n) // 32], s_g[off // 32:(off + n) // 32]
            # group scales follow the f32 values: a few ulps apart (the rmsnorm sum of
            # squares is a tree sum here, sequential on the CPU)
            srel = float(np.max(np.abs(sg.astype(np.float64) - so) / np.abs(so)))
            assert srel <= 1e-5, f"{name} pos {pos}: scales differ by {srel:.1e}"
            total += n
            if np.any(d):
                assert np.max(np.abs(d)) <= 1, f"{name} pos {pos}: int8 activations differ by >1 (a bug, not a flip)"
                idx = np.nonzero(d)[0]
                t = v_o[off + idx].astype(np.float64) / np.repeat(so, 32)[idx]
                tie = np.abs(np.abs(t - np.trunc(t)) - 0.5)
                assert np.all(tie < 1e-3), f"{name} pos {pos}: a flip away from a rounding tie ({tie.max():.2e})"
                flips += int(idx.size)
                first = off
        if first is None:
            assert rel(lg_g, lg_o) < LOGIT_TOL, f"{name} pos {pos}: no flip but logits differ"
            if margin(lg_o) > LOGIT_TOL:
                assert int(np.argmax(lg_g)) == int(np.argmax(lg_o))
        else:
            flip_steps += 1
            assert rel(lg_g, lg_o) < 5e-2
    # Every flip was proven a rounding tie above, and flipped elements stay a small
    # minority.  Steps with a flip can be common: Q4_0 embedding rows put whole
    # groups on exact ties at the first layer's input, so only require that some
    # steps went end-to-end flip-free and had their logits checked at LOGIT_TOL.
    assert flip_steps < steps, f"{name}: every step had a rounding flip"
    assert flips <= max(32, total // 100), f"{name}: {flips} flipped activations of {total}"


@pytest.mark.parametrize("name", ["llama_q8", "qwen2_mix", "llama_kq"])
def test_prefill_then_decode(models, name):
    _, om, gm = models[name]
    rng = np.random.default_rng(6)
    toks = rng.integers(gm.config.vocab_size, size=21).astype(np.uint32)
    okv, gkv = om.kv(40), pm.KvCache(gm, 40)
    om.prefill(okv, toks)
    pm.prefill(gm, gkv, toks)
    ref = om.forward(okv, 9, len(toks))
    got, _ = pm.forward(gm, gkv, 9, len(toks))
    assert rel(got, ref) < FREE_TOL


@pytest.mark.parametrize("name", ["llama_q8", "qwen2_mix"])
@pytest.mark.parametrize("n", [1, 5, 8, 11])
def test_forward_batch(models, name, n):
    _, om, gm = models[name]
    rng = np.random.default_rng(7)
    pre = rng.integers(gm.config.vocab_size, size=6).astype(np.uint32)
    toks = rng.integers(gm.config.vocab_size, size=n).astype(np.uint32)
    okv, gkv = om.kv(40), pm.KvCache(gm, 40)
    om.prefill(okv, pre)
    pm.prefill(gm, gkv, pre)
    ref = om.forward_batch(okv, toks, len(pre))
    got, am = pm.forward_batch(gm, gkv, toks, len(pre))
    assert rel(got, ref) < FREE_TOL
    assert np.array_equal(am, np.argmax(got, axis=1))


@pytest.mark.parametrize("name", list(SPECS))
def test_generate_greedy_tokens(models, name):
    path, om, gm = models[name]
    rng = np.random.default_rng(8)
    prompt = rng.integers(gm.config.vocab_size, size=8).astype(np.uint32)
    steps = 40
    ref = om.generate(prompt, steps)
    got = pm.generate(gm, prompt, steps)
    assert len(got) == len(ref)
    # identical up to the first position whose oracle top-2 margin is within tolerance
    okv = om.kv(len(prompt) + steps)
    om.prefill(okv, prompt[:-1])
    tok = int(prompt[-1])
    for i in range(len(ref)):
        lg = om.forward(okv, tok, len(prompt) - 1 + i)
        if margin(lg) <= FREE_TOL:
            break
        assert got[i] == ref[i], f"{name}: token {i} differs with margin {margin(lg):.2e}"
        tok = int(ref[i])


def test_generate_speculative_equals_greedy(models):
    """generate_speculative emits exactly the target's greedy sequence (gguf.rs:745-846)."""
    _, _, target = models["qwen2_mix"]
    _, _, draft_self = models["qwen2_mix"]
    _, _, draft_other = models["llama_q8"]
    rng = np.random.default_rng(9)
    prompt = rng.integers(min(target.config.vocab_size, draft_other.config.vocab_size), size=6).astype(np.uint32)
    plain = pm.generate(target, prompt, 30)
    spec, (proposed, accepted) = pm.generate_speculative(target, draft_self, prompt, 30, 4)
    assert np.array_equal(spec, plain)
    assert accepted > 0 and proposed >= accepted


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
