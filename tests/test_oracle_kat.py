"""The CPU oracle against the reference's own known-answer tests (CPU only).

Each test restates one test of the Prana workspace with the same inputs and
the same assertions, so the oracle that checks the CUDA library is itself
pinned to the reference's published behaviour:

  f16 conversions      crates/prana-kernels/src/lib.rs:119-154, crates/prana-model/src/gguf.rs:887-897
  block formats        crates/prana-model/src/gguf.rs:929-1070
  native vs dequant    crates/prana-kernels/src/kquant.rs:385-477 (pseudo_bytes seeds)
  SIMD == scalar       crates/prana-kernels/src/kquant.rs:479-523
  matmul               crates/prana-kernels/src/matmul.rs:412-470
  norms / activations  crates/prana-kernels/src/norms.rs:62-109
  rope / attention     crates/prana-kernels/src/attention.rs:339-502
"""
import math
import struct

import numpy as np
import pytest

F16_ONE = 0x3C00
M64 = (1 << 64) - 1


def pseudo_bytes(n: int, seed: int) -> np.ndarray:
    """The reference tests' xorshift byte stream (kquant.rs:385-395)."""
    s = max(seed, 1)
    out = np.empty(n, np.uint8)
    for i in range(n):
        s ^= s >> 12
        s ^= (s << 25) & M64
        s ^= s >> 27
        out[i] = ((s * 0x2545F4914F6CDD1D) & M64) >> 56
    return out


def f32s(x):
    return np.asarray(x, np.float32)


# ------------------------------------------------------------------ f16 (lib.rs:119-154, gguf.rs:887-897)

def test_f16_exact_values_round_trip(oracle):
    for v in [0.0, -0.0, 1.0, -1.0, 0.5, 2.0, -2.0, 0.25, 65504.0, -65504.0]:
        back = oracle.f16_to_f32(oracle.f32_to_f16(v))
        assert struct.pack("<f", back) == struct.pack("<f", v), v


def test_f16_rounds_to_nearest_and_stays_close(oracle):
    for i in range(-2000, 2000):
        v = float(np.float32(i) * np.float32(0.0017))
        r = oracle.f16_to_f32(oracle.f32_to_f16(v))
        assert abs(r - v) <= abs(v) * 1e-3 + 1e-6, (v, r)


def test_f16_specials_and_overflow(oracle):
    assert oracle.f32_to_f16(math.inf) == 0x7C00
    assert oracle.f32_to_f16(-math.inf) == 0xFC00
    assert math.isnan(oracle.f16_to_f32(oracle.f32_to_f16(math.nan)))
    assert oracle.f32_to_f16(1e30) == 0x7C00
    assert oracle.f32_to_f16(1e-30) == 0x0000


def test_f16_ties_to_even(oracle):
    assert oracle.f32_to_f16(1.0 + 2.0 ** -11) == 0x3C00


def test_f16_to_f32_cases(oracle):
    assert oracle.f16_to_f32(0x0000) == 0.0
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xC000) == -2.0
    assert oracle.f16_to_f32(0x7C00) == math.inf
    assert math.isnan(oracle.f16_to_f32(0x7E00))
    assert abs(oracle.f16_to_f32(0x0001) - 2.0 ** -24) < 1e-12
    assert abs(oracle.f16_to_f32(0x3555) - 0.33325) < 1e-4


# ------------------------------------------------------------------ block formats (gguf.rs:929-1070)

def test_q4k_block_known_values(oracle):
    b = np.zeros(144, np.uint8)
    b[0:2] = np.frombuffer(struct.pack("<H", F16_ONE), np.uint8)  # d = 1
    b[4], b[5] = 2, 3  # group scales 2, 3
    for i in range(32):
        b[16 + i] = (i % 16) | ((15 - i % 16) << 4)
    out = np.empty(256, np.float32)
    oracle.lib().or_dequant_q4k_block(oracle.ptr(b), oracle.ptr(out))
    for i in range(32):
        assert out[i] == 2.0 * (i % 16)
        assert out[32 + i] == 3.0 * (15 - i % 16)
    assert np.all(out[64:] == 0.0)


def test_q4k_packed_scale_min_high_groups(oracle):
    import ctypes

    s = np.zeros(12, np.uint8)
    s[8] = (53 & 0xF) | ((43 & 0xF) << 4)
    s[0] = (53 >> 4) << 6
    s[4] = (43 >> 4) << 6
    sc, m = ctypes.c_float(), ctypes.c_float()
    oracle.lib().or_q4k_scale_min(4, oracle.ptr(s), ctypes.byref(sc), ctypes.byref(m))
    assert (sc.value, m.value) == (53.0, 43.0)


def test_q6k_block_known_values(oracle):
    b = np.zeros(210, np.uint8)
    b[192:208] = 1
    b[208:210] = np.frombuffer(struct.pack("<H", F16_ONE), np.uint8)
    b[0] = 5
    b[128] = 2
    out = np.empty(256, np.float32)
    oracle.lib().or_dequant_q6k_block(oracle.ptr(b), oracle.ptr(out))
    assert out[0] == 5 + (2 << 4) - 32
    assert out[1] == -32.0
    assert out[64] == -32.0


def _q4_0_row():
    raw = bytearray(struct.pack("<H", F16_ONE))
    raw += bytes(j | ((15 - j) << 4) for j in range(16))
    raw += struct.pack("<H", 0x3800)  # d = 0.5
    raw += bytes([0xCC] * 16)
    return np.frombuffer(bytes(raw), np.uint8)


def test_q4_0_dequant_and_native_dot(oracle):
    m = oracle.OMatrix(2, 1, 64, _q4_0_row())
    f = m.dequant()[0]
    for j in range(16):
        assert f[j] == j - 8.0
        assert f[16 + j] == (15 - j) - 8.0
    assert np.all(f[32:] == 0.5 * (12.0 - 8.0))
    x = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.37)).astype(np.float32)
    want = float(np.dot(x.astype(np.float64), f))
    got = float(m.matmul(x)[0, 0])
    assert abs(got - want) < 2e-2 * max(abs(want), 1.0)


def test_q8_0_row_dot(oracle):
    raw = struct.pack("<H", F16_ONE) + bytes((i - 16) & 0xFF for i in range(32))
    m = oracle.OMatrix(8, 1, 32, np.frombuffer(raw, np.uint8))
    assert abs(float(m.matmul(np.ones(32, np.float32))[0, 0]) + 16.0) < 1e-4


# ------------------------------------------------------------------ native vs dequant (kquant.rs:385-477)

KINDS = {"q4_0": (2, 18, 32), "q4_k": (12, 144, 256), "q6_k": (14, 210, 256)}


def _random_blocks(kind, n_blocks, seed):
    t, bb, _ = KINDS[kind]
    b = pseudo_bytes(n_blocks * bb, seed).reshape(n_blocks, bb)
    if kind == "q4_0":
        b[:, 0:2] = (0x66, 0x2E)  # d ~ 0.1
    elif kind == "q4_k":
        b[:, 0:2] = (0x66, 0x2E)
        b[:, 2:4] = (0x66, 0x2A)  # dmin ~ 0.05
    else:
        b[:, 208:210] = (0x66, 0x2E)
    return b.reshape(-1)


@pytest.mark.parametrize("kind,seed", [("q4_0", 3), ("q4_0", 77), ("q4_0", 2024), ("q4_k", 1), ("q4_k", 42),
                                       ("q4_k", 12345), ("q6_k", 7), ("q6_k", 99), ("q6_k", 54321)])
def test_native_matmul_matches_dequant_reference(oracle, kind, seed):
    t, bb, bv = KINDS[kind]
    rows, cols, n_tokens = 5, 512, 2
    m = oracle.OMatrix(t, rows, cols, _random_blocks(kind, rows * cols // bv, seed))
    a = np.sin(np.arange(n_tokens * cols, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    native = m.matmul(a, oracle.TIER_SCALAR)
    a_dq = []
    for row in a.reshape(n_tokens, cols):
        q, s, _ = oracle.quantize_acts(row)
        a_dq.append(q.astype(np.float32) * np.repeat(s, 32))
    dense = np.stack(a_dq).astype(np.float64) @ m.dequant().astype(np.float64).T
    tol = 1e-3 * np.maximum(np.abs(dense), 1.0)
    assert np.all(np.abs(native - dense) < tol)


def test_q40_row_dequant_matches_full(oracle):
    rows, cols = 3, 64
    m = oracle.OMatrix(2, rows, cols, _random_blocks("q4_0", rows * cols // 32, 9))
    full = m.dequant()
    for r in range(rows):
        row = np.empty(cols, np.float32)
        oracle.lib().or_matrix_dequant_row.argtypes = [oracle.P, oracle.SZ, oracle.P]
        oracle.lib().or_matrix_dequant_row(oracle.C.byref(m.m), r, oracle.ptr(row))
        assert np.array_equal(row, full[r])


@pytest.mark.parametrize("kind", ["q4_0", "q4_k"])
def test_simd_dots_match_scalar(oracle, kind):
    if not oracle.lib().or_simd_available():
        pytest.skip("no AVX2+FMA on this CPU")
    t, bb, bv = KINDS[kind]
    cols = 512
    m = oracle.OMatrix(t, 1, cols, _random_blocks(kind, cols // bv, 31 + bb))
    a = np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.021)).astype(np.float32)
    scalar = float(m.matmul(a, oracle.TIER_SCALAR)[0, 0])
    tiers = [oracle.TIER_AVX2] + ([oracle.TIER_VNNI] if oracle.lib().or_vnni_available() and kind == "q4_0" else [])
    for tier in tiers:
        simd = float(m.matmul(a, tier)[0, 0])
        assert abs(scalar - simd) < 1e-3 * max(abs(scalar), 1.0), (tier, scalar, simd)


# ------------------------------------------------------------------ matmul (matmul.rs:412-470)

def test_f32_matmul_matches_reference(oracle):
    a = f32s([1, 2, 3, 4, 5, 6])
    w = f32s([1, 0, 0, 0, 1, 0, 0, 0, 1, 1, 1, 1])
    m = oracle.OMatrix(0, 4, 3, w)
    assert m.matmul(a).reshape(-1).tolist() == [1, 2, 3, 6, 4, 5, 6, 15]


def _quantize_q8(oracle, w, rows, cols):
    q = np.empty(rows * cols, np.int8)
    s = np.empty(rows * cols // 32, np.float32)
    oracle.lib().or_quantize_q8(rows, cols, oracle.ptr(np.ascontiguousarray(w, np.float32)), oracle.ptr(q),
                                oracle.ptr(s))
    return q, s


def test_q8_roundtrip_is_close(oracle):
    rows, cols = 8, 64
    w = np.sin(np.arange(rows * cols, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    q, s = _quantize_q8(oracle, w, rows, cols)
    dq = q.astype(np.float32) * np.repeat(s, 32)
    assert float(np.max(np.abs(w - dq))) < 0.01
    assert q.nbytes + s.nbytes < w.nbytes


def _q8_gguf(q, s):
    """int8 + f32 scales -> GGUF Q8_0 bytes (f16 d), scales taken f16-exact."""
    out = bytearray()
    for g in range(s.size):
        out += struct.pack("<e", float(s[g])) + q[g * 32:(g + 1) * 32].tobytes()
    return np.frombuffer(bytes(out), np.uint8)


def test_q8_matmul_tracks_f32(oracle):
    n_rows, k = 6, 96
    a = np.cos(np.arange(k, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w = np.sin(np.arange(n_rows * k, dtype=np.float32) * np.float32(0.017)).astype(np.float32)
    dense = oracle.OMatrix(0, n_rows, k, w).matmul(a)
    q, s = _quantize_q8(oracle, w, n_rows, k)
    quant = oracle.OMatrix(8, n_rows, k, _q8_gguf(q, s)).matmul(a)
    assert np.all(np.abs(dense - quant) < 0.05)


def test_prefill_and_decode_agree(oracle):
    n_rows, k = 5, 32
    w = np.sin(np.arange(n_rows * k, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    batch = np.cos(np.arange(3 * k, dtype=np.float32) * np.float32(0.011)).astype(np.float32)
    m = oracle.OMatrix(0, n_rows, k, w)
    allr = m.matmul(batch)
    for t in range(3):
        assert np.array_equal(allr[t], m.matmul(batch[t * k:(t + 1) * k])[0])


# ------------------------------------------------------------------ norms (norms.rs:62-109)

def test_rmsnorm_unit_weight_normalizes(oracle):
    x, w, y = f32s([2, 2, 2, 2]), f32s([1, 1, 1, 1]), np.empty(4, np.float32)
    oracle.lib().or_rmsnorm(oracle.ptr(x), oracle.ptr(w), 1, 4, 0.0, oracle.ptr(y))
    assert np.all(np.abs(y - 1.0) < 1e-5)


def _softmax(oracle, x):
    x = f32s(x)
    out = np.empty_like(x)
    oracle.lib().or_softmax(oracle.ptr(x), x.size, oracle.ptr(out))
    return out


def test_softmax_sums_to_one_and_is_overflow_safe(oracle):
    p = _softmax(oracle, [1, 2, 3])
    assert abs(float(p.sum()) - 1.0) < 1e-6 and p[0] < p[1] < p[2]
    p = _softmax(oracle, [1000, 1001])
    assert np.all(np.isfinite(p)) and abs(float(p.sum()) - 1.0) < 1e-6


def test_silu_matches_definition(oracle):
    x = f32s([0, 1, -1, 4])
    oracle.lib().or_silu(oracle.ptr(x), 4)
    assert x[0] == 0.0
    assert abs(x[1] - 0.7310586) < 1e-5
    assert abs(x[2] + 0.2689414) < 1e-5
    assert 3.9 < x[3] < 4.0


# ------------------------------------------------------------------ rope / attention (attention.rs:339-502)

def _rope_batch(oracle, x, seq, nh, hd, theta=10000.0):
    oracle.lib().or_rope_batch(oracle.ptr(x), seq, nh, hd, theta)


def test_rope_preserves_pair_norm(oracle):
    seq, nh, hd = 3, 2, 4
    x = (np.sin(np.arange(seq * nh * hd, dtype=np.float32) * np.float32(0.1)) + np.float32(0.3)).astype(np.float32)
    before = x.copy()
    _rope_batch(oracle, x, seq, nh, hd)
    half = hd // 2
    for p in range(seq):
        for h in range(nh):
            base = (p * nh + h) * hd
            for j in range(half):
                n0 = before[base + j] ** 2 + before[base + j + half] ** 2
                n1 = x[base + j] ** 2 + x[base + j + half] ** 2
                assert abs(n0 - n1) < 1e-5


def test_rope_identity_at_position_zero(oracle):
    x = np.arange(8, dtype=np.float32)
    before = x.copy()
    _rope_batch(oracle, x, 1, 1, 8)
    assert np.all(np.abs(x - before) < 1e-6)


def test_rope_interleaved_pos0_identity_and_pair_norm(oracle):
    hd = 8
    x = (np.sin(np.arange(2 * hd, dtype=np.float32) * np.float32(0.3)) + np.float32(0.1)).astype(np.float32)
    before = x.copy()
    oracle.lib().or_rope_interleaved(oracle.ptr(x), x.size, 0, hd, 10000.0)
    assert np.array_equal(x, before)
    oracle.lib().or_rope_interleaved(oracle.ptr(x), x.size, 7, hd, 10000.0)
    for i in range(0, x.size, 2):
        assert abs((before[i] ** 2 + before[i + 1] ** 2) - (x[i] ** 2 + x[i + 1] ** 2)) < 1e-4


def test_rope_neox_matches_batch_rope(oracle):
    nh, hd = 2, 8
    w = nh * hd
    row = (np.sin(np.arange(w, dtype=np.float32) * np.float32(0.17)) + np.float32(0.2)).astype(np.float32)
    pos = 3
    batch = np.zeros(4 * w, np.float32)
    batch[pos * w:(pos + 1) * w] = row
    _rope_batch(oracle, batch, 4, nh, hd)
    single = row.copy()
    oracle.lib().or_rope_neox(oracle.ptr(single), w, pos, hd, 10000.0)
    assert np.all(np.abs(single - batch[pos * w:(pos + 1) * w]) < 1e-5)


def _attention(oracle, q, k, v, seq, nh, nkv, hd):
    out = np.empty(seq * nh * hd, np.float32)
    oracle.lib().or_attention(oracle.ptr(q), oracle.ptr(k), oracle.ptr(v), seq, nh, nkv, hd, oracle.ptr(out))
    return out


def test_attention_pos0_returns_v0(oracle):
    seq, nh, hd = 4, 2, 3
    n = seq * nh * hd
    q = np.cos(np.arange(n, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    k = np.sin(np.arange(n, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    v = np.cos(np.arange(n, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    out = _attention(oracle, q, k, v, seq, nh, nh, hd)
    assert np.all(np.abs(out[:nh * hd] - v[:nh * hd]) < 1e-5)


def test_attention_output_bounded_by_v_range(oracle):
    seq, hd = 5, 4
    q = np.sin(np.arange(seq * hd, dtype=np.float32) * np.float32(0.2)).astype(np.float32)
    k = np.cos(np.arange(seq * hd, dtype=np.float32) * np.float32(0.15)).astype(np.float32)
    v = np.sin(np.arange(seq * hd, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    out = _attention(oracle, q, k, v, seq, 1, 1, hd)
    for i in range(seq):
        vis = v[:(i + 1) * hd]
        o = out[i * hd:(i + 1) * hd]
        assert np.all(o >= vis.min() - 1e-5) and np.all(o <= vis.max() + 1e-5)


def test_decode_with_cache_matches_full_attention(oracle):
    seq, nh, hd = 5, 2, 4
    w = nh * hd
    q = np.sin(np.arange(seq * w, dtype=np.float32) * np.float32(0.07)).astype(np.float32)
    k = np.cos(np.arange(seq * w, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    v = np.sin(np.arange(seq * w, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    full = _attention(oracle, q, k, v, seq, nh, nh, hd)
    kh = np.array([oracle.f32_to_f16(float(x)) for x in k], np.uint16)
    vh = np.array([oracle.f32_to_f16(float(x)) for x in v], np.uint16)
    for pos in range(seq):
        step = np.empty(w, np.float32)
        qp = np.ascontiguousarray(q[pos * w:(pos + 1) * w])
        oracle.lib().or_attention_decode(oracle.ptr(qp), oracle.ptr(kh), oracle.ptr(vh), pos, nh, nh, hd,
                                         oracle.ptr(step))
        assert np.all(np.abs(full[pos * w:(pos + 1) * w] - step) < 3e-3)


def test_grouped_query_attention_shapes(oracle):
    seq, nh, nkv, hd = 3, 4, 2, 2
    q = (np.arange(seq * nh * hd, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    k = (np.arange(seq * nkv * hd, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    v = (np.arange(seq * nkv * hd, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    out = _attention(oracle, q, k, v, seq, nh, nkv, hd)
    assert out.size == seq * nh * hd and np.all(np.isfinite(out))
