"""GPU parity of every kernel-level entry point against the CPU oracle.

Integer work (activation quantization, per-block int8 dots, f16 KV writes,
RoPE with the shared host table, argmax) must be bit-exact.  Float
accumulations differ only in summation order: tolerances are stated per test
(normwise relative error = max|gpu - oracle| / max|oracle|).
"""
import numpy as np
import pytest
import torch

from prana_b200 import kernels as K
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu

TYPES = [TYPE_Q8_0, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K]
GEMV_TOL = 2e-5  # normwise, f32 accumulation order only


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def acts(seed, rows, k, scale=1.0):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((rows, k)) * scale).astype(np.float32)
    a[:, :32] = 0.0  # an all-zero group (scale 1.0 path)
    if rows > 1:
        a[1, 32:64] = np.float32(3.0e4)  # saturating group
    return a


def test_quantize_acts_bit_exact(gpu, oracle):
    a = acts(1, 7, 4096, 2.5)
    qa = K.quantize_acts(cuda(a))
    torch.cuda.synchronize()
    for r in range(a.shape[0]):
        q, s, sm = oracle.quantize_acts(a[r])
        assert np.array_equal(qa.q[r].cpu().numpy(), q)
        assert np.array_equal(qa.scales[r].cpu().numpy().view(np.uint32), s.view(np.uint32))
        assert np.array_equal(qa.sums[r].cpu().numpy(), sm)


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("k", [256, 768, 4096])
def test_block_dots_bit_exact(gpu, oracle, ty, k):
    rows = 5
    w = synth.matrix(ty, rows, k, seed=11 + ty, std=0.02)
    gw = K.QuantMatrix(ty, rows, k, w)
    a = acts(2, 1, k)
    qa = K.quantize_acts(cuda(a))
    q, s, sm = oracle.quantize_acts(a[0])
    for r in range(rows):
        got = K.block_dots(gw, r, qa).cpu().numpy()
        # the oracle's Q8_0 row is the int8 plane (QuantMatrix layout, matmul.rs:21-30)
        row = np.ascontiguousarray(w[r].reshape(-1, 34)[:, 2:]).reshape(-1) if ty == TYPE_Q8_0 else w[r]
        ref = oracle.block_dots(ty, q, row, k)
        assert np.array_equal(got, ref), f"type {ty} row {r}"


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("n_tokens", [1, 2, 3, 5, 8, 13])
def test_gemv_matches_oracle(gpu, oracle, ty, n_tokens):
    rows, k = 300, 1024
    w = synth.matrix(ty, rows, k, seed=3 + ty)
    gw = K.QuantMatrix(ty, rows, k, w)
    om = oracle.OMatrix(ty, rows, k, w)
    a = acts(5 + n_tokens, n_tokens, k)
    ref = om.matmul(a, oracle.TIER_SCALAR)
    fn = K.matmul_q8_f32 if ty == TYPE_Q8_0 else K.matmul_kquant_f32
    got = fn(cuda(a), gw, n_tokens).cpu().numpy()
    assert rel(got, ref) < GEMV_TOL


@pytest.mark.parametrize("ty", TYPES)
def test_gemv_prefill_matches_oracle(gpu, oracle, ty):
    rows, k, n = 129, 2048, 11
    w = synth.matrix(ty, rows, k, seed=21 + ty)
    gw = K.QuantMatrix(ty, rows, k, w)
    om = oracle.OMatrix(ty, rows, k, w)
    a = acts(9, n, k)
    q, s, sm = oracle.quantize_acts_rows(a)
    ref = om.matmul_prefill(q, s, sm, oracle.TIER_SCALAR)
    qa = K.QuantActs(cuda(q), cuda(s), cuda(sm))
    fn = K.matmul_q8_prefill if ty == TYPE_Q8_0 else K.matmul_kquant_prefill
    got = fn(qa, gw).cpu().numpy()
    assert rel(got, ref) < GEMV_TOL


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("n_tokens", [6, 8])
def test_matmul_tall_weight_tensor_cores(gpu, oracle, ty, n_tokens):
    """6-8 rows against a weight of >= 8192 rows take the tensor-core GEMM at
    kernel level (the GEMV's cost grows with the rows, the GEMM's does not);
    Q6_K stays on the GEMV."""
    rows, k = 8200, 1024
    w = synth.matrix(ty, rows, k, seed=50 + ty + n_tokens)
    gw = K.QuantMatrix(ty, rows, k, w)
    om = oracle.OMatrix(ty, rows, k, w)
    a = acts(60 + n_tokens, n_tokens, k)
    ref = om.matmul(a, oracle.TIER_SCALAR)
    fn = K.matmul_q8_f32 if ty == TYPE_Q8_0 else K.matmul_kquant_f32
    got = fn(cuda(a), gw, n_tokens).cpu().numpy()
    assert rel(got, ref) < GEMV_TOL


def test_gemv_large_rows(gpu, oracle):
    """Shapes of the 8B microbench at K=4096 (rows trimmed for oracle time)."""
    for ty in TYPES:
        rows, k = 1031, 4096
        w = synth.matrix(ty, rows, k, seed=99)
        gw = K.QuantMatrix(ty, rows, k, w)
        om = oracle.OMatrix(ty, rows, k, w)
        a = np.random.default_rng(0).standard_normal((1, k)).astype(np.float32)
        fn = K.matmul_q8_f32 if ty == TYPE_Q8_0 else K.matmul_kquant_f32
        assert rel(fn(cuda(a), gw, 1).cpu().numpy(), om.matmul(a, oracle.TIER_SCALAR)) < GEMV_TOL


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("k", [768, 4096])
def test_gemv_batch1_pipeline(gpu, oracle, ty, k):
    """Batch 1 with enough rows that every warp streams whole rows (no K split):
    the double-buffered path that walks (row group, chunk) items, including
    rows of several chunks (K = 4096) and rows shorter than one warp's chunk."""
    rows = 2402
    w = synth.matrix(ty, rows, k, seed=400 + ty + k)
    gw = K.QuantMatrix(ty, rows, k, w)
    om = oracle.OMatrix(ty, rows, k, w)
    a = np.random.default_rng(k).standard_normal((1, k)).astype(np.float32)
    fn = K.matmul_q8_f32 if ty == TYPE_Q8_0 else K.matmul_kquant_f32
    assert rel(fn(cuda(a), gw, 1).cpu().numpy(), om.matmul(a, oracle.TIER_SCALAR)) < GEMV_TOL


def test_rmsnorm(gpu, oracle):
    import ctypes as C

    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 896)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(896)).astype(np.float32)
    ref = np.empty_like(x)
    oracle.lib().or_rmsnorm(oracle.ptr(x), oracle.ptr(w), 3, 896, C.c_float(1e-6), oracle.ptr(ref))
    got = K.rmsnorm(cuda(x), cuda(w), 3, 896, 1e-6).cpu().numpy()
    assert rel(got, ref) < 1e-6


@pytest.mark.parametrize("neox", [False, True])
def test_rope_bit_exact(gpu, oracle, neox):
    import ctypes as C

    hd, heads, pos = 64, 4, 37
    rng = np.random.default_rng(6)
    x = rng.standard_normal((3, heads * hd)).astype(np.float32)
    ref = x.copy()
    for r in range(3):
        row = np.ascontiguousarray(ref[r])
        fn = oracle.lib().or_rope_neox if neox else oracle.lib().or_rope_interleaved
        fn(oracle.ptr(row), row.size, pos + r, hd, C.c_float(1e6 if neox else 1e4))
        ref[r] = row
    g = cuda(x)
    (K.rope_neox if neox else K.rope_interleaved)(g, pos, hd, 1e6 if neox else 1e4)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_silu_softmax_argmax(gpu, oracle):
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(5000) * 4).astype(np.float32)
    ref = x.copy()
    oracle.lib().or_silu(oracle.ptr(ref), ref.size)
    g = cuda(x)
    K.silu(g)
    assert rel(g.cpu().numpy(), ref) < 1e-6
    sref = np.empty_like(x)
    oracle.lib().or_softmax(oracle.ptr(x), x.size, oracle.ptr(sref))
    assert rel(K.softmax(cuda(x)).cpu().numpy(), sref) < 1e-5
    x[[17, 4000]] = 100.0  # tie: first index wins
    assert int(K.argmax(cuda(x)).cpu()[0]) == 17 == oracle.lib().or_argmax(oracle.ptr(x), x.size)


def test_f16_kv_write_bit_exact(gpu, oracle):
    rng = np.random.default_rng(10)
    src = np.concatenate([rng.standard_normal(1000).astype(np.float32) * 100,
                          np.array([1e30, -1e30, 1e-30, 65504.0, 1.0 + 2 ** -11, 6e-8], np.float32)])
    cache = torch.zeros(4 * 1006, dtype=torch.int16, device="cuda")
    K.f16_kv_write(cache, 2, 1006, cuda(src))
    got = cache.cpu().numpy().view(np.uint16)[2 * 1006:3 * 1006]
    ref = np.array([oracle.f32_to_f16(float(v)) for v in src], np.uint16)
    assert np.array_equal(got, ref)


def _cache(seed, rows, kv_dim):
    rng = np.random.default_rng(seed)
    f = rng.standard_normal((rows, kv_dim)).astype(np.float32)
    return np.array([[0]], np.uint16) if rows == 0 else f.astype(np.float16).view(np.uint16)


# tensor-core path: hd 64/128 with <= 16 query heads per kv head; CUDA-core path otherwise
@pytest.mark.parametrize("nh,nkv,hd,pos", [(6, 6, 48, 0), (6, 6, 48, 255), (14, 2, 64, 2047), (32, 8, 128, 700),
                                           (12, 2, 128, 1023), (32, 8, 128, 4095), (8, 1, 64, 5), (4, 4, 64, 16),
                                           (4, 4, 64, 129), (64, 2, 128, 300), (16, 16, 32, 77),
                                           # one rank's shard of the 8B shape at 8, 4 and 2 GPUs
                                           (4, 1, 128, 4095), (8, 2, 128, 4095), (16, 4, 128, 4095)])
def test_attention_decode(gpu, oracle, nh, nkv, hd, pos):
    kc = _cache(1, pos + 1, nkv * hd)
    vc = _cache(2, pos + 1, nkv * hd)
    q = np.random.default_rng(3).standard_normal(nh * hd).astype(np.float32)
    ref = np.empty(nh * hd, np.float32)
    oracle.lib().or_attention_decode(oracle.ptr(q), oracle.ptr(kc), oracle.ptr(vc), pos, nh, nkv, hd, oracle.ptr(ref))
    got = K.attention_decode(cuda(q), cuda(kc.view(np.int16)), cuda(vc.view(np.int16)), pos, nh, nkv, hd).cpu().numpy()
    assert rel(got, ref) < 2e-5


@pytest.mark.parametrize("nh,nkv,hd,seq", [(6, 6, 48, 5), (14, 2, 64, 5), (12, 2, 128, 5), (32, 8, 128, 8),
                                           (8, 1, 64, 3)])
def test_attention_verify(gpu, oracle, nh, nkv, hd, seq):
    pos0 = 300
    kc = _cache(4, pos0 + seq, nkv * hd)
    vc = _cache(5, pos0 + seq, nkv * hd)
    q = np.random.default_rng(6).standard_normal((seq, nh * hd)).astype(np.float32)
    ref = np.empty_like(q)
    oracle.lib().or_attention_verify(oracle.ptr(q), oracle.ptr(kc), oracle.ptr(vc), pos0, seq, nh, nkv, hd, oracle.ptr(ref))
    got = K.attention_verify(cuda(q), cuda(kc.view(np.int16)), cuda(vc.view(np.int16)), pos0, seq, nh, nkv, hd).cpu().numpy()
    assert rel(got, ref) < 2e-5


@pytest.mark.parametrize("nh,nkv,hd,seq,qscale", [(6, 6, 48, 7, 1.0), (14, 2, 64, 300, 1.0), (32, 8, 128, 130, 1.0),
                                                  (14, 2, 64, 1100, 1.0), (8, 8, 32, 200, 4.0), (12, 4, 96, 77, 1.0),
                                                  (4, 2, 256, 40, 1.0), (16, 2, 128, 257, 3.0), (3, 1, 64, 1, 1.0)])
def test_attention_prefill(gpu, oracle, nh, nkv, hd, seq, qscale):
    """Causal prefill attention over f32 in-window K/V: rows that end inside a
    key tile, partial CTAs, one row, sharp softmaxes (qscale) and the CUDA-core
    kernel at head dim 256."""
    rng = np.random.default_rng(7)
    q = (qscale * rng.standard_normal((seq, nh * hd))).astype(np.float32)
    k = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    ref = np.empty_like(q)
    oracle.lib().or_attention(oracle.ptr(q), oracle.ptr(k), oracle.ptr(v), seq, nh, nkv, hd, oracle.ptr(ref))
    got = K.attention(cuda(q), cuda(k), cuda(v), seq, nh, nkv, hd).cpu().numpy()
    assert rel(got, ref) < 2e-5


def test_quantize_acts_nan_is_zero(gpu, oracle):
    """A NaN activation quantizes to 0 (Rust's clamp keeps the NaN, `as` makes it
    0) and leaves its group's scale to the other values (matmul.rs:109-126)."""
    a = acts(3, 2, 256)
    a[0, 40] = np.nan
    a[1, 100] = np.nan
    qa = K.quantize_acts(cuda(a))
    torch.cuda.synchronize()
    for r in range(2):
        q, s, sm = oracle.quantize_acts(a[r])
        assert np.array_equal(qa.q[r].cpu().numpy(), q)
        assert np.array_equal(qa.scales[r].cpu().numpy().view(np.uint32), s.view(np.uint32))
        assert np.array_equal(qa.sums[r].cpu().numpy(), sm)
