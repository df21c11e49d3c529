"""quantize_q8 (matmul.rs:61-84) in the library's host code against the oracle
(CPU only): int8 values and f32 scales bit for bit, including all-zero blocks
(scale 1), saturating values, half-way cases of the rounding and NaN."""
import numpy as np

from prana_b200 import kernels as K


def test_quantize_q8_bit_exact(oracle):
    rng = np.random.default_rng(3)
    rows, cols = 37, 256
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0                                  # all-zero block: scale 1
    w[1, :32] = np.float32(3e4)                      # saturating block
    w[2, :32] = np.arange(32, dtype=np.float32) - 15.5  # halves: round away from zero
    w[3, 5] = np.nan                                 # NaN: 0, as `as i8`
    q, s = K.quantize_q8(rows, cols, w)
    qo = np.empty(rows * cols, np.int8)
    so = np.empty(rows * cols // 32, np.float32)
    oracle.lib().or_quantize_q8(rows, cols, oracle.ptr(w.reshape(-1)), oracle.ptr(qo), oracle.ptr(so))
    assert np.array_equal(q.reshape(-1), qo)
    assert np.array_equal(s.reshape(-1).view(np.uint32), so.view(np.uint32))
    assert s[0, 0] == 1.0 and q[3, 5] == 0
