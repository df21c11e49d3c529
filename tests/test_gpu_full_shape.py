"""Parity at the benchmarked configuration's full width (GPU).

The decode benchmark runs the Llama-3-8B shape (dim 4096, 32 query / 8 kv
heads of 128, FFN 14336, vocab 128256) over an f16 KV cache holding 4096
positions, in Q4_0 and Q8_0.  These tests run exactly those tensor shapes --
every projection, the full-vocabulary LM head, attention over 4096 cached
positions -- with 2 layers instead of 32 so the CPU oracle keeps up, and
check 8 consecutive decode steps teacher-forced from the oracle's cache:
every int8 activation row equal up to rounding ties, logits within 1e-3, the
greedy token wherever the top-2 margin exceeds 1e-3 (tests/parity.py).  The
KV rows are the benchmark's seeded N(0, 0.5) f16 rows.
"""
import numpy as np
import pytest

from oracle.parity import Flips, check_logits, forced_decode
from prana_b200 import model as pm
from prana_b200 import synth

pytestmark = pytest.mark.gpu

CTX = 4096
STEPS = 8


def seeded_kv_rows(layer, is_v, rows, kv_dim, seed=4242):
    """The benchmark's cache contents (bench.py seeds the same way)."""
    rng = np.random.default_rng([seed, layer, int(is_v)])
    return (rng.standard_normal((rows, kv_dim), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("preset", ["llama3_8b_q4_0_l2", "llama3_8b_q8_0_l2"])
def test_full_width_decode_at_ctx_4096(tmp_path, gpu, oracle, preset):
    spec = synth.PRESETS[preset]
    path = tmp_path / f"{preset}.gguf"
    synth.write_gguf(spec, path)
    om = oracle.OModel(str(path), oracle.TIER_AUTO)
    gm = pm.Model.load(str(path), 0)
    try:
        c = gm.config
        assert (c.dim, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden_dim, c.vocab_size) == \
            (4096, 32, 8, 128, 14336, 128256)
        kv_dim = c.n_kv_heads * c.head_dim
        okv, gkv = om.kv(CTX + STEPS), pm.KvCache(gm, CTX + STEPS)
        for layer in range(c.n_layers):
            for is_v in (False, True):
                okv.set_layer(layer, is_v, seeded_kv_rows(layer, is_v, CTX, kv_dim))
        flips, gated = Flips(), 0
        tok = 17
        for i in range(STEPS):
            pos = CTX + i
            for layer in range(c.n_layers):
                for is_v in (False, True):
                    gkv.write(layer, is_v, okv.layer(layer, is_v)[:pos])
            lg_g, lg_o = forced_decode(om, okv, gm, gkv, tok, pos, flips, f"{preset} pos {pos}")
            gated += check_logits(lg_g, lg_o, f"{preset} pos {pos}")
            # the CUDA-graph decode step computes the traced pass's logits
            lg_p, nxt = pm.forward(gm, gkv, tok, pos)
            assert np.array_equal(lg_p, lg_g) and nxt == int(np.argmax(lg_g))
            tok = int(np.argmax(lg_o))
        assert flips.bounded(), f"{flips.flips} flipped activations of {flips.total}"
        assert gated >= STEPS // 2
        gkv.close()
    finally:
        gm.close()
