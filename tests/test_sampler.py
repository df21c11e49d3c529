"""The host sampler against the reference's sampler tests (sampler.rs:72-106)
and, draw for draw, against a restatement that takes its softmax from the C
oracle (norms.rs:44-56) and its uniform draws from xorshift64* written out
here (sampler.rs:51-70).  CPU only."""
import numpy as np

from oracle import oracle as orc
from prana_b200.sampler import Sampler

MASK = 2**64 - 1


class XorShift:
    def __init__(self, seed):
        self.s = max(seed, 1)

    def next_f32(self):
        x = self.s
        x ^= x >> 12
        x ^= (x << 25) & MASK
        x ^= x >> 27
        self.s = x
        v = (x * 0x2545F4914F6CDD1D) & MASK
        return np.float32(v >> 40) / np.float32(1 << 24)


def test_greedy_picks_the_max():
    assert Sampler(0.0, 42).sample([0.1, 3.0, -1.0, 2.9]) == 1
    assert Sampler(0.0, 1).sample([2.0, 5.0, 5.0]) == 1  # the first maximum


def test_temperature_sampling_is_seeded_and_in_range():
    logits = [1.0, 2.0, 3.0, 4.0]
    a, b = Sampler(0.8, 7), Sampler(0.8, 7)
    for _ in range(50):
        x, y = a.sample(logits), b.sample(logits)
        assert x == y and 0 <= x < len(logits)


def test_rng_is_roughly_uniform():
    s = Sampler(1.0, 123)
    draws = np.array([s.next_f32() for _ in range(10_000)], dtype=np.float64)
    assert abs(draws.mean() - 0.5) < 0.02


def test_draws_match_the_restatement_exactly():
    rng = np.random.default_rng(3)
    logits = (rng.standard_normal(3000) * 3).astype(np.float32)
    for temp, seed in [(0.7, 11), (1.0, 0), (1.5, 2**63 + 5)]:
        s, ref = Sampler(temp, seed), XorShift(seed)
        scaled = logits / np.float32(temp)
        probs = np.empty_like(scaled)
        orc.lib().or_softmax(scaled.ctypes.data, scaled.size, probs.ctypes.data)
        for _ in range(200):
            r = ref.next_f32()
            want = len(probs) - 1
            for i, p in enumerate(probs):
                r = np.float32(r - p)
                if r <= 0:
                    want = i
                    break
            assert s.sample(logits) == want


def test_nan_temperature_samples_like_the_reference():
    """Sampler::new takes the temperature branch unless temp <= 0 (sampler.rs:14),
    so a NaN temperature samples: every scaled logit is NaN, no bucket takes the
    draw and the last id comes back, one draw consumed."""
    s = Sampler(float("nan"), 5)
    assert s.sample([1.0, 2.0, 3.0]) == 2
    ref = XorShift(5)
    ref.next_f32()
    assert np.float32(s.next_f32()) == ref.next_f32()


def test_oracle_sampler_matches_host_sampler():
    """The oracle's or_sample (the checker of the device sampler) against the
    host sampler, draw for draw, including non-finite rows."""
    rng = np.random.default_rng(8)
    rows = [(rng.standard_normal(5000) * 2).astype(np.float32),
            np.where(np.arange(700) % 4 == 0, -np.inf, rng.standard_normal(700)).astype(np.float32)]
    bad = rows[0].copy()
    bad[17] = np.nan
    rows.append(bad)
    for logits in rows:
        for temp, seed in [(0.8, 7), (1.2, 0)]:
            s, o = Sampler(temp, seed), orc.OSampler(temp, seed)
            for _ in range(50):
                assert s.sample(logits) == o.sample(logits)[0]
            assert s.next_f32() == o.next_f32()
    assert orc.OSampler(0.0, 3).sample(np.array([1, 5, 5, 2], np.float32))[0] == 1
