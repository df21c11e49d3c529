"""The oracle's activation trace and its forced mode (CPU only).

Forcing a pass with its own trace must change nothing: the matmuls then take
the rows they would have quantized themselves, through matmul_*_prefill,
whose per-element dot is the decode GEMV's (matmul.rs:185-232,
kquant.rs:368-370).  The batch trace of a verify pass must equal the
sequential single-token passes row for row (forward_batch and forward_impl
run the same per-row arithmetic, infer.rs:142-211 / 296-374)."""
import numpy as np
import pytest

from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

SPECS = {
    "llama_q8": synth.ModelSpec("llama", 128, 256, 2, 4, 2, 32, 300, 64, 10000.0, 1e-5, seed=21),
    "qwen2_mix": synth.ModelSpec("qwen2", 256, 512, 2, 4, 1, 64, 400, 64, 1e6, 1e-6, has_bias=True, seed=22,
                                 type_embd=TYPE_Q4_0, type_q=TYPE_Q4_K, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                                 type_o=TYPE_Q4_0, type_gate=TYPE_Q4_K, type_up=TYPE_Q4_K, type_down=TYPE_Q6_K,
                                 type_output=TYPE_Q8_0),
}


@pytest.fixture(scope="module", params=list(SPECS))
def om(request, tmp_path_factory, oracle):
    path = tmp_path_factory.mktemp("trace") / f"{request.param}.gguf"
    synth.write_gguf(SPECS[request.param], path)
    return oracle.OModel(str(path), oracle.TIER_SCALAR)


def test_forced_with_own_trace_changes_nothing(om):
    kv1, kv2 = om.kv(8), om.kv(8)
    for pos, tok in enumerate([3, 17, 5]):
        lg, q, s = om.forward_trace(kv1, tok, pos)
        lg2, q2, s2 = om.forward_trace(kv2, tok, pos, force=(q, s))
        assert np.array_equal(lg, lg2) and np.array_equal(q, q2) and np.array_equal(s, s2)


def test_batch_trace_forced_with_own_trace_changes_nothing(om):
    toks = np.array([4, 9, 2, 7, 1], np.uint32)
    for verify in (False, True):
        kv1, kv2 = om.kv(16), om.kv(16)
        if verify:
            om.prefill(kv1, toks[:3])
            om.prefill(kv2, toks[:3])
        lg, q, s = om.batch_trace(kv1, toks, 3 if verify else 0, verify)
        lg2, q2, s2 = om.batch_trace(kv2, toks, 3 if verify else 0, verify, force=(q, s))
        assert np.array_equal(q, q2) and np.array_equal(s, s2)
        if verify:
            assert np.array_equal(lg, lg2)
        for layer in range(om.c.n_layers):
            for is_v in (False, True):
                assert np.array_equal(kv1.layer(layer, is_v), kv2.layer(layer, is_v))


def test_verify_rows_equal_sequential_passes(om):
    pre = np.array([6, 8, 10], np.uint32)
    toks = np.array([4, 9, 2, 7], np.uint32)
    kvb, kvs = om.kv(16), om.kv(16)
    om.prefill(kvb, pre)
    om.prefill(kvs, pre)
    lg, q, s = om.batch_trace(kvb, toks, len(pre), True)
    c = om.c
    per = [c.dim, c.n_heads * c.head_dim, c.dim, c.hidden_dim]
    n = len(toks)
    for i, t in enumerate(toks):
        lgi, qi, si = om.forward_trace(kvs, int(t), len(pre) + i)
        assert np.array_equal(lgi, lg[i])
        # site by site: row i of the batch site equals the single pass's site
        off_b = off_s = 0
        for _ in range(c.n_layers):
            for k in per:
                assert np.array_equal(q[off_b + i * k: off_b + (i + 1) * k], qi[off_s: off_s + k])
                off_b += n * k
                off_s += k
        assert np.array_equal(q[off_b + i * c.dim: off_b + (i + 1) * c.dim], qi[off_s: off_s + c.dim])
