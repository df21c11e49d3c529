"""Dense tensors under the reference's two precisions (GPU).

gguf::load(path, precision) (gguf.rs:338-460) keeps GGUF Q8_0/Q4_0/Q4_K/Q6_K
tensors packed and turns dense ones (F32, F16) into Linear::new(w, precision):
quantize_q8 (matmul.rs:61-84) under Q8, the dense f32 matmul under F32.  A tied
classifier over a densified embedding table (F32, F16, Q8_0) is quantize_q8 of
the table under Q8 and the dense f32 head (matmul_f32) under F32
(gguf.rs:425-437, checkpoint.rs:239-248).  Each case is checked against the
oracle loaded at the same precision, through the forced parity check
(oracle/parity.py): logits within 1e-3, the greedy token wherever the top-2
margin exceeds 1e-3.
"""
import numpy as np
import pytest
import torch

from oracle.parity import Flips, check_logits, forced_batch, forced_decode, rel
from prana_b200 import kernels as K
from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_F16, TYPE_F32, TYPE_Q4_0, TYPE_Q8_0

pytestmark = pytest.mark.gpu

CASES = {
    # tied Q8_0 table, F32 precision: the dense f32 classifier over the densified table
    "tied_q8_table_f32": (synth.ModelSpec("llama", 256, 512, 2, 8, 4, 32, 900, 64, 1e4, 1e-5, tied=True, seed=61),
                          pm.PRECISION_F32),
    # tied F16 table, Q8 precision: quantize_q8 of the table
    "tied_f16_table_q8": (synth.ModelSpec("qwen2", 256, 512, 2, 4, 1, 64, 700, 64, 1e6, 1e-6, has_bias=True, tied=True,
                                          seed=62, type_embd=TYPE_F16, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0,
                                          type_v=TYPE_Q8_0, type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0,
                                          type_down=TYPE_Q8_0), pm.PRECISION_Q8),
    # dense F32 projections and head, Q8 precision: every matrix is quantize_q8 of it
    "dense_f32_q8": (synth.ModelSpec("llama", 256, 512, 2, 8, 4, 32, 600, 64, 1e4, 1e-5, seed=63).with_types(TYPE_F32),
                     pm.PRECISION_Q8),
}


@pytest.fixture(scope="module")
def models(tmp_path_factory, gpu, oracle):
    d = tmp_path_factory.mktemp("precision")
    out = {}
    for name, (spec, prec) in CASES.items():
        path = d / f"{name}.gguf"
        synth.write_gguf(spec, path)
        out[name] = (oracle.OModel(str(path), oracle.TIER_SCALAR, prec), pm.Model.load(str(path), 0, precision=prec))
    yield out
    for _, gm in out.values():
        gm.close()


@pytest.mark.parametrize("name", list(CASES))
def test_decode_forced(models, name):
    om, gm = models[name]
    c = gm.config
    okv, gkv = om.kv(20), pm.KvCache(gm, 20)
    flips, gated = Flips(), 0
    rng = np.random.default_rng(4)
    for pos in range(12):
        tok = int(rng.integers(c.vocab_size))
        lg_g, lg_o = forced_decode(om, okv, gm, gkv, tok, pos, flips, f"{name} pos {pos}")
        gated += check_logits(lg_g, lg_o, f"{name} pos {pos}")
        lg_p, nxt = pm.forward(gm, gkv, tok, pos)  # the CUDA-graph step computes the traced pass's logits
        assert np.array_equal(lg_p, lg_g) and nxt == int(np.argmax(lg_g))
    assert flips.bounded() and gated >= 6


@pytest.mark.parametrize("name", list(CASES))
def test_batch_forced(models, name):
    """forward_batch above 8 rows (the tensor-core path for the quantize_q8
    matrices; 8-row f32 GEMV launches for the dense classifier)."""
    om, gm = models[name]
    c = gm.config
    rng = np.random.default_rng(5)
    pre = rng.integers(c.vocab_size, size=5).astype(np.uint32)
    toks = rng.integers(c.vocab_size, size=11).astype(np.uint32)
    okv, gkv = om.kv(24), pm.KvCache(gm, 24)
    flips = Flips()
    forced_batch(om, okv, gm, gkv, pre, 0, True, flips, f"{name} prefill")
    lg_g, lg_o = forced_batch(om, okv, gm, gkv, toks, len(pre), False, flips, f"{name} verify")
    for i in range(len(toks)):
        check_logits(lg_g[i], lg_o[i], f"{name} row {i}")


def test_generate_and_decode_loop(models):
    """The device decode loop with the dense classifier (argmax kernel, token
    fed back through a device copy) generates what the step entry point does."""
    _, gm = models["tied_q8_table_f32"]
    prompt = np.array([3, 14, 15, 92], np.uint32)
    got = pm.generate(gm, prompt, 12)
    kv = pm.KvCache(gm, 32)
    pm.prefill(gm, kv, prompt[:-1])
    tok, ref = int(prompt[-1]), []
    for i in range(12):
        _, tok = pm.forward(gm, kv, tok, len(prompt) - 1 + i)
        ref.append(tok)
    assert np.array_equal(got, np.array(ref, np.uint32))


@pytest.mark.parametrize("m", [1, 3, 8, 20])
def test_quantize_q8_weight_matmul(gpu, oracle, m):
    """Linear::new(w, Q8): a quantize_q8 weight through matmul_q8_f32 (the GEMV
    up to 8 rows, the tensor cores above) against the oracle's."""
    rng = np.random.default_rng(m)
    rows, cols = 300, 1024
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    gw = K.QuantMatrix.quantize_q8(rows, cols, w)
    a = rng.standard_normal((m, cols)).astype(np.float32)
    got = K.matmul_q8_f32(torch.from_numpy(a).cuda(), gw, m).cpu().numpy()
    ref = oracle.OQ8Matrix(rows, cols, w).matmul(a, oracle.TIER_SCALAR)
    assert rel(got, ref) < 2e-5
    # per-block int32 dots of the quantize_q8 matrix are the reference's
    qa = K.quantize_acts(torch.from_numpy(a).cuda())
    q, _ = K.quantize_q8(rows, cols, w)
    for r in (0, 77, rows - 1):
        dots = K.block_dots(gw, r, qa).cpu().numpy()
        ref_d = oracle.block_dots(TYPE_Q8_0, qa.q[0].cpu().numpy(), q[r], cols)
        assert np.array_equal(dots, ref_d)
