"""The tensor-core GEMM (tcgen05 kind::i8, prana_qgemm) against the CPU oracle.

Every 32-value block (16 for Q6_K) is one MMA into a fresh TMEM accumulator,
so the per-block int32 dots must equal the reference's scalar dots bit for bit
(dot_q8_q8_scalar, matmul.rs:395-406; dot_q40_q8_scalar, dot_q4k_q8_scalar,
dot_q6k_q8_scalar, kquant.rs:240-318) at every row / token / block, including
partial weight tiles (rows not a multiple of 128), partial token tiles and K
not a multiple of the 256-value stage.  The f32 results must match the
oracle's matmul_*_prefill (matmul.rs:185-232, kquant.rs:368-370) within the
GEMV tolerance (f32 summation order only).
"""
import numpy as np
import pytest
import torch

from prana_b200 import kernels as K
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu

TOL = 2e-5  # normwise, f32 accumulation order only


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def acts(seed, rows, k):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((rows, k)).astype(np.float32)
    a[:, :32] = 0.0  # an all-zero group
    if rows > 1:
        a[1, 32:64] = np.float32(3.0e4)  # a saturating group
    return a


def oracle_row(ty, w, r):
    # the oracle's Q8_0 row is the int8 plane (QuantMatrix layout, matmul.rs:21-30)
    return np.ascontiguousarray(w[r].reshape(-1, 34)[:, 2:]).reshape(-1) if ty == TYPE_Q8_0 else w[r]


CASES = [
    # (type, K, N, M)
    (TYPE_Q8_0, 1024, 200, 1), (TYPE_Q8_0, 896, 130, 17), (TYPE_Q8_0, 288, 256, 40), (TYPE_Q8_0, 4096, 256, 64),
    (TYPE_Q4_0, 1024, 200, 3), (TYPE_Q4_0, 896, 130, 16), (TYPE_Q4_0, 288, 128, 33), (TYPE_Q4_0, 4096, 384, 64),
    (TYPE_Q4_K, 1024, 200, 5), (TYPE_Q4_K, 768, 130, 20), (TYPE_Q4_K, 4096, 256, 64),
    (TYPE_Q6_K, 1024, 200, 2), (TYPE_Q6_K, 768, 130, 31), (TYPE_Q6_K, 4096, 256, 64),
]


@pytest.mark.parametrize("ty,k,n,m", CASES)
def test_block_dots_bit_exact(gpu, oracle, ty, k, n, m):
    w = synth.matrix(ty, n, k, seed=100 + ty + k + n)
    gw = K.QuantMatrix(ty, n, k, w)
    a = acts(7 + m, m, k)
    qa = K.quantize_acts(torch.from_numpy(a).cuda())
    got = K.qgemm_block_dots(qa, gw).cpu().numpy()
    q = qa.q.cpu().numpy()
    # every token against a spread of rows, including the last partial tile
    rows = sorted(set(list(range(0, n, max(1, n // 9))) + [n - 1]))
    for t in range(m):
        for r in rows:
            ref = oracle.block_dots(ty, q[t], oracle_row(ty, w, r), k)
            assert np.array_equal(got[t, r], ref), f"type {ty} token {t} row {r}"


@pytest.mark.parametrize("ty,k,n,m", CASES)
def test_values_match_oracle_prefill(gpu, oracle, ty, k, n, m):
    w = synth.matrix(ty, n, k, seed=200 + ty + k + n)
    gw = K.QuantMatrix(ty, n, k, w)
    a = acts(9 + m, m, k)
    qa = K.quantize_acts(torch.from_numpy(a).cuda())
    got = K.qgemm(qa, gw).cpu().numpy()
    om = oracle.OMatrix(ty, n, k, w)
    ref = om.matmul_prefill(qa.q.cpu().numpy(), qa.scales.cpu().numpy(), qa.sums.cpu().numpy(), oracle.TIER_SCALAR)
    assert got.shape == ref.shape
    assert rel(got, ref) < TOL


@pytest.mark.parametrize("ty", [TYPE_Q8_0, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K])
def test_full_width_shape(gpu, oracle, ty):
    """The 8B FFN shape [14336 x 4096] at 64 rows, sampled against the oracle."""
    n, k, m = 14336, 4096, 64
    w = synth.matrix(ty, n, k, seed=300 + ty)
    gw = K.QuantMatrix(ty, n, k, w)
    a = acts(11, m, k)
    qa = K.quantize_acts(torch.from_numpy(a).cuda())
    got = K.qgemm(qa, gw).cpu().numpy()
    rows = np.arange(0, n, 97)
    om = oracle.OMatrix(ty, len(rows), k, np.ascontiguousarray(w[rows]))
    ref = om.matmul_prefill(qa.q.cpu().numpy(), qa.scales.cpu().numpy(), qa.sums.cpu().numpy(), oracle.TIER_SCALAR)
    assert rel(got[:, rows], ref) < TOL


def test_repeated_calls_are_identical(gpu):
    """TMEM is freed and the barriers reset between launches: ten calls agree bitwise."""
    n, k, m = 640, 2048, 48
    w = synth.matrix(TYPE_Q4_0, n, k, seed=5)
    gw = K.QuantMatrix(TYPE_Q4_0, n, k, w)
    qa = K.quantize_acts(torch.randn(m, k, device="cuda"))
    first = K.qgemm(qa, gw)
    for _ in range(9):
        assert torch.equal(K.qgemm(qa, gw), first)
    K.synchronize()
