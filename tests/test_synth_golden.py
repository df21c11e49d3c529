"""Seeded-model encoders against the reference's own K-quant encoders (CPU only).

tests/golden/kquant_encode.npz holds seeded f32 blocks and the Q4_K / Q6_K
super-blocks that the reference's scripts/convert-to-gguf.py:29-89
(`q4k_encode_block`, `q6k_encode_block`) produced for them; make_golden.py in
that folder regenerates it from a reference checkout.  The encoders that write
this repository's synthetic GGUF models must reproduce every byte, and the
oracle must decode the blocks back within the formats' quantization step.
"""
from pathlib import Path

import numpy as np
import pytest

from prana_b200 import build as pbuild
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_K, TYPE_Q6_K

GOLDEN = Path(__file__).resolve().parent / "golden" / "kquant_encode.npz"


@pytest.fixture(scope="module")
def golden():
    if not synth.LIB_PATH.exists():
        pbuild.build_synth()
    return np.load(GOLDEN)


@pytest.mark.parametrize("ggml_type,key", [(TYPE_Q4_K, "q4_k"), (TYPE_Q6_K, "q6_k")])
def test_encoder_matches_reference_bytes(golden, ggml_type, key):
    x, want = golden["x"], golden[key]
    got = synth.encode(ggml_type, x)
    bad = [i for i in range(len(x)) if not np.array_equal(got[i], want[i])]
    assert not bad, f"{key}: blocks {bad} differ from the reference encoder"


@pytest.mark.parametrize("ggml_type,key", [(TYPE_Q4_K, "q4_k"), (TYPE_Q6_K, "q6_k")])
def test_reference_blocks_decode_close(oracle, golden, ggml_type, key):
    x, blocks = golden["x"], golden[key]
    m = oracle.OMatrix(ggml_type, len(x), 256, blocks.reshape(-1))
    y = m.dequant()
    # per-block error bounded by the block's range over the format's levels
    span = np.maximum(np.max(np.abs(x), axis=1, keepdims=True), 1e-6)
    levels = 15.0 if key == "q4_k" else 31.0
    assert np.all(np.abs(y - x) <= span * (2.5 / levels) + 1e-5)
