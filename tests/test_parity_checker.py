"""The forced parity checker (tests/parity.py) on the CPU, without a GPU.

The reference's AVX2/VNNI tier sums its dots in another order than its scalar
tier, exactly the kind of difference the GPU path has; run against each other
through the forced check, the two tiers must pass at the north-star
tolerance.  A mistake planted in one side's activation rows, scales or K/V
rows must be caught."""
import numpy as np
import pytest

from oracle.parity import Flips, check_logits, check_trace
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q6_K, TYPE_Q8_0

SPEC = synth.ModelSpec("qwen2", 256, 512, 2, 4, 1, 64, 500, 64, 1e6, 1e-6, has_bias=True, seed=51,
                       type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                       type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                       type_output=TYPE_Q8_0)


@pytest.fixture(scope="module")
def tiers(tmp_path_factory, oracle):
    if not oracle.lib().or_simd_available():
        pytest.skip("no AVX2 on this host")
    path = tmp_path_factory.mktemp("tiers") / "m.gguf"
    synth.write_gguf(SPEC, path)
    return oracle.OModel(str(path), oracle.TIER_SCALAR), oracle.OModel(str(path), oracle.TIER_AVX2)


def kv_rows(okv, n_layers, first, n):
    return np.concatenate([okv.layer(l, v)[first:first + n].reshape(-1) for l in range(n_layers) for v in (False, True)])


def step(ref, other, rkv, okv, tok, pos, flips, plant=None):
    c = ref.c
    lg_x, q_x, s_x = other.forward_trace(okv, tok, pos)
    kv_x = kv_rows(okv, c.n_layers, pos, 1)
    if plant:
        q_x, s_x, kv_x = plant(q_x.copy(), s_x.copy(), kv_x.copy())
    lg_r, q_r, s_r, v_r, kv_r, kv_v = ref.forward_trace(rkv, tok, pos, with_values=True, force=(q_x, s_x),
                                                         force_kv=kv_x)
    flips.check_kv(kv_x, kv_r, kv_v, f"pos {pos}", c.n_kv_heads * c.head_dim)
    check_trace(c, q_x, s_x, q_r, s_r, v_r, flips, f"pos {pos}")
    return check_logits(lg_x, lg_r, f"pos {pos}")


def test_tiers_agree_through_the_forced_check(tiers):
    ref, other = tiers
    rkv, okv = ref.kv(24), other.kv(24)
    flips, gated = Flips(), 0
    rng = np.random.default_rng(3)
    for pos in range(20):
        gated += step(ref, other, rkv, okv, int(rng.integers(ref.c.vocab_size)), pos, flips)
    assert flips.bounded() and gated >= 10


@pytest.mark.parametrize("what", ["int8", "scale", "kv"])
def test_planted_mistake_is_caught(tiers, what):
    ref, other = tiers
    rkv, okv = ref.kv(8), other.kv(8)

    def plant(q, s, kv):
        if what == "int8":
            q[300] = np.int8(int(q[300]) + 3 if q[300] < 100 else int(q[300]) - 3)
        elif what == "scale":
            s[5] *= np.float32(1.01)
        else:
            kv[17] ^= np.uint16(0x0100)  # a few f16 ulps off
        return q, s, kv

    for pos in range(2):
        step(ref, other, rkv, okv, 7 + pos, pos, Flips())
    with pytest.raises(AssertionError):
        step(ref, other, rkv, okv, 11, 2, Flips(), plant=plant)
