"""Temperature sampling on the device (Sampler::sample, sampler.rs:22-37)
against the CPU oracle's restatement, draw for draw from the same seeded
xorshift64* stream: the same id, or -- where the ids differ -- a draw that lies
at every bucket boundary between them within the reference's own sequential
f32 rounding (oracle.parity.sample_boundary_gap).  Then generate with a sampler
and the sampled device decode loop, teacher-forced against the oracle."""
import zlib

import numpy as np
import pytest
import torch

from oracle.parity import sample_boundary_gap
from prana_b200 import kernels as K
from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import PranaError
from prana_b200.sampler import Sampler

pytestmark = pytest.mark.gpu


def run_draws(oracle, logits: np.ndarray, temp: float, seed: int, draws: int):
    """Device and oracle ids for `draws` draws over one row; returns the number
    of differing ids (each one checked against the boundary rule)."""
    dev = torch.from_numpy(logits).cuda()
    s, o = Sampler(temp, seed), oracle.OSampler(temp, seed)
    diffs = 0
    for i in range(draws):
        got = int(K.sample(s, dev).item())
        want, probs, r = o.sample(logits)
        assert 0 <= got < logits.size
        if got != want:
            diffs += 1
            a, b = min(got, want), max(got, want)
            gap = sample_boundary_gap(probs, r, a, b)
            assert gap <= 0, f"draw {i}: device {got}, oracle {want}, r={r}: boundary off by {gap:.3g}"
    # the host stream skipped exactly the draws the kernel took
    assert s.next_f32() == o.next_f32()
    return diffs


SHAPES = [
    ("flat_llama3", 128256, lambda g, n: g.normal(0, 1, n)),
    ("peaked_llama3", 128256, lambda g, n: g.normal(0, 3, n) + np.where(np.arange(n) % 9973 == 5, 25.0, 0.0)),
    ("qwen2_vocab", 151936, lambda g, n: g.standard_t(3, n) * 2),
    ("stories", 32000, lambda g, n: g.normal(0, 2, n)),
    ("small", 7, lambda g, n: g.normal(0, 1, n)),
    ("one", 1, lambda g, n: g.normal(0, 1, n)),
    ("ragged", 1031, lambda g, n: g.normal(0, 1, n)),
    ("masked", 5000, lambda g, n: np.where(np.arange(n) % 3 == 0, -np.inf, g.normal(0, 1, n))),
]


@pytest.mark.parametrize("name,n,gen", SHAPES, ids=[s[0] for s in SHAPES])
@pytest.mark.parametrize("temp", [0.5, 0.8, 1.0, 1.7])
def test_sample_matches_oracle(gpu, oracle, name, n, gen, temp):
    g = np.random.default_rng(zlib.crc32(f"{name}/{temp}".encode()))
    logits = gen(g, n).astype(np.float32)
    diffs = run_draws(oracle, logits, temp, seed=int(g.integers(1, 2**63)), draws=40)
    if n <= 1031:  # short rows: the reference's own rounding moves no boundary far
        assert diffs <= 1, f"{diffs} of 40 draws differ"


def test_sample_greedy_and_seed_zero(gpu, oracle):
    logits = np.array([0.1, 3.0, -1.0, 3.0, 2.9], np.float32)
    dev = torch.from_numpy(logits).cuda()
    assert int(K.sample(Sampler(0.0, 42), dev).item()) == 1  # the first maximum
    assert int(K.sample(Sampler(-1.0, 42), dev).item()) == 1
    # a zero seed reads as 1 (XorShift::new)
    assert run_draws(oracle, logits, 0.9, seed=0, draws=20) == 0


def test_sample_non_finite(gpu, oracle):
    """A NaN or +inf logit makes every probability 0 or NaN in the reference:
    the running draw never reaches 0 and the last id is taken."""
    g = np.random.default_rng(3)
    for bad in (np.nan, np.inf):
        logits = g.normal(0, 1, 4096).astype(np.float32)
        logits[100] = bad
        dev = torch.from_numpy(logits).cuda()
        s, o = Sampler(0.8, 11), oracle.OSampler(0.8, 11)
        for _ in range(5):
            want = o.sample(logits)[0]
            assert int(K.sample(s, dev).item()) == want == logits.size - 1
    # a NaN temperature samples (Sampler::new only tests temperature <= 0)
    logits = g.normal(0, 1, 300).astype(np.float32)
    s, o = Sampler(float("nan"), 5), oracle.OSampler(float("nan"), 5)
    assert int(K.sample(s, torch.from_numpy(logits).cuda()).item()) == o.sample(logits)[0] == 299


def test_sample_largest_vocab_and_limit(gpu, oracle):
    n = 8 * 49152
    logits = np.random.default_rng(9).normal(0, 1.5, n).astype(np.float32)
    run_draws(oracle, logits, 0.8, seed=77, draws=8)
    with pytest.raises(PranaError):
        K.sample(Sampler(0.8, 1), torch.zeros(n + 1, device="cuda"))


SPEC = synth.ModelSpec("llama", 256, 512, 3, 8, 4, 32, 1000, 160, 10000.0, 1e-5, seed=1)


@pytest.fixture(scope="module")
def small_model(tmp_path_factory, gpu, oracle):
    path = tmp_path_factory.mktemp("sample") / "m.gguf"
    synth.write_gguf(SPEC, path)
    gm = pm.Model.load(str(path), 0)
    yield path, oracle.OModel(str(path), oracle.TIER_SCALAR), gm
    gm.close()


def replay_sampled(oracle, om, prompt, toks, temp, seed):
    """Teacher-forced oracle replay of a sampled generation: at each step the
    oracle samples from its own logits with its own stream; a differing id must
    sit at a bucket boundary within the logits tolerance.  Returns the oracle's
    stream state and the number of differing ids."""
    kv = om.kv(len(prompt) + len(toks) + 1)
    if len(prompt) > 1:
        om.prefill(kv, prompt[:-1])
    o = oracle.OSampler(temp, seed)
    tok, pos, diffs = int(prompt[-1]), len(prompt) - 1, 0
    for want_dev in toks:
        lg = om.forward(kv, tok, pos)
        want, probs, r = o.sample(lg)
        if want != int(want_dev):
            diffs += 1
            a, b = min(want, int(want_dev)), max(want, int(want_dev))
            # the GPU's logits may differ by the logits tolerance (1e-3 of the
            # largest): allow that much probability at the boundary
            assert sample_boundary_gap(probs, r, a, b, tol=1e-3) <= 0, f"pos {pos}: {want_dev} vs {want}"
        tok, pos = int(want_dev), pos + 1
    return o, diffs


@pytest.mark.parametrize("temp,seed", [(0.8, 7), (1.0, 12345), (1.3, 0)])
def test_generate_sampled_matches_oracle(small_model, oracle, temp, seed):
    _, om, gm = small_model
    prompt = np.array([1, 17, 250, 3, 999], np.uint32)
    s = Sampler(temp, seed)
    toks = pm.generate_sampled(gm, prompt, 40, s)
    assert toks.size == 40
    o, diffs = replay_sampled(oracle, om, prompt, toks, temp, seed)
    assert diffs <= 2
    # the caller's sampler continues exactly where the reference's would
    assert s.next_f32() == o.next_f32()
    # the oracle's own sampled generate gives the same ids where nothing differed
    if diffs == 0:
        want, _ = om.generate_sampled(prompt, 40, temp, seed)
        assert np.array_equal(toks, want)


def test_generate_sampled_stop_token(small_model, oracle):
    """Stopping on a sampled stop id leaves the sampler one draw past it."""
    _, om, gm = small_model
    prompt = np.array([5, 6, 7], np.uint32)
    full = pm.generate_sampled(gm, prompt, 30, Sampler(0.9, 99))
    stop = int(full[10])
    first = int(np.nonzero(full == stop)[0][0])
    s = Sampler(0.9, 99)
    got = pm.generate_sampled(gm, prompt, 30, s, stop_id=stop)
    assert np.array_equal(got, full[:first])
    ref = Sampler(0.9, 99)
    for _ in range(first + 1):
        ref.next_f32()
    assert s.next_f32() == ref.next_f32()


def test_decode_loop_sampled(small_model):
    """The sampled device loop replays the same draws as generate_sampled, and a
    greedy sampler gives the greedy loop (caches sized as generate sizes its own)."""
    _, _, gm = small_model
    prompt = np.array([1, 17, 250, 3, 999], np.uint32)
    for steps, sampler, want in ((24, Sampler(0.8, 7), pm.generate_sampled(gm, prompt, 24, Sampler(0.8, 7))),
                                 (12, Sampler(0.0, 7), pm.generate(gm, prompt, 12))):
        kv = pm.KvCache(gm, len(prompt) + steps)
        pm.prefill(gm, kv, prompt[:-1])
        loop = pm.DecodeLoop(gm, kv)
        loop.begin(int(prompt[-1]), len(prompt) - 1, sampler=sampler)
        loop.run(steps)
        assert np.array_equal(loop.tokens(steps), want)
        kv.close()


def test_forward_sampled_matches_loop(small_model):
    """Token by token (prana_forward_sampled) the draws are the sampled loop's,
    and the sampler ends where generate_sampled leaves it."""
    _, _, gm = small_model
    prompt = np.array([1, 17, 250, 3, 999], np.uint32)
    s_loop = Sampler(0.7, 31)
    want = pm.generate_sampled(gm, prompt, 20, s_loop)
    kv = pm.KvCache(gm, len(prompt) + 20)
    pm.prefill(gm, kv, prompt[:-1])
    s = Sampler(0.7, 31)
    tok, got = int(prompt[-1]), []
    for pos in range(len(prompt) - 1, len(prompt) - 1 + 20):
        tok = pm.forward_sampled(gm, kv, tok, pos, s)
        got.append(tok)
    kv.close()
    assert np.array_equal(np.array(got, np.uint32), want)
    assert s.next_f32() == s_loop.next_f32()
