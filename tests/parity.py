"""Shared parity checks of the GPU model path against the CPU oracle.

The GPU quantizes the same f32 activations as the CPU path, but its f32 sums
run in another order (tree reductions, per-lane partial sums), so a value that
sits within ~1e-6 of a rounding boundary of `quantize_acts` (matmul.rs:109-126)
can land one int8 step apart.  The reference's own scalar and AVX2/VNNI tiers
differ the same way.  The checks here therefore run the oracle in forced mode:
at every quantization site it records its own int8 rows, proves that each
difference from the GPU's rows is such a rounding tie, and then continues with
the GPU's rows.  Downstream values then differ only by summation order, so the
logits of every step can be held to the north-star tolerance (1e-3 max
relative error) and the greedy token must match wherever the top-2 margin
exceeds it.
"""
from __future__ import annotations

import numpy as np

LOGIT_TOL = 1e-3   # max |gpu - oracle| / max |oracle| (BASELINE logits tolerance)
TIE_TOL = 1e-3     # a flipped element's x / scale lies within this of k + 1/2
SCALE_TOL = 1e-5   # per-32 scales follow the f32 values (a few ulps)


def rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def margin(lg) -> float:
    s = np.sort(np.asarray(lg, np.float64))
    return float((s[-1] - s[-2]) / max(float(np.max(np.abs(lg))), 1e-30))


def site_lengths(c, rows: int = 1, final: bool = True):
    """(length of one row, rows) of every trace site in forward order."""
    out = []
    for _ in range(c.n_layers):
        for k in (c.dim, c.n_heads * c.head_dim, c.dim, c.hidden_dim):
            out.append((k, rows))
    if final:
        out.append((c.dim, rows))
    return out


class Flips:
    """Running count of int8 rounding flips and compared elements."""

    def __init__(self):
        self.flips = 0
        self.total = 0

    def check(self, q_g, s_g, q_o, s_o, v_o, where: str) -> None:
        """Every element of the GPU's rows equals the oracle's, or differs by one
        step at a rounding tie of the oracle's own value; scales agree."""
        q_g = np.asarray(q_g)
        q_o = np.asarray(q_o)
        assert q_g.shape == q_o.shape
        srel = float(np.max(np.abs(np.asarray(s_g, np.float64) - s_o) / np.maximum(np.abs(s_o), 1e-30)))
        assert srel <= SCALE_TOL, f"{where}: scales differ by {srel:.1e}"
        d = q_g.astype(np.int32) - q_o
        self.total += d.size
        if not np.any(d):
            return
        assert np.max(np.abs(d)) <= 1, f"{where}: int8 activations differ by more than one step"
        idx = np.nonzero(d)[0]
        t = np.asarray(v_o, np.float64)[idx] / np.repeat(np.asarray(s_o, np.float64), 32)[idx]
        tie = np.abs(np.abs(t - np.trunc(t)) - 0.5)
        assert np.all(tie < TIE_TOL), f"{where}: a flip away from a rounding tie ({tie.max():.2e})"
        self.flips += int(idx.size)

    def bounded(self, frac: float = 0.01, floor: int = 32) -> bool:
        return self.flips <= max(floor, int(self.total * frac))


def check_trace(c, q_g, s_g, q_o, s_o, v_o, flips: Flips, where: str, rows: int = 1, final: bool = True):
    off = 0
    for i, (k, r) in enumerate(site_lengths(c, rows, final)):
        n = k * r
        flips.check(q_g[off:off + n], s_g[off // 32:(off + n) // 32], q_o[off:off + n],
                    s_o[off // 32:(off + n) // 32], v_o[off:off + n], f"{where} site {i}")
        off += n
    assert off == len(q_g)


def check_logits(lg_g, lg_o, where: str) -> bool:
    """Logits within LOGIT_TOL; returns whether the greedy token was gated in."""
    r = rel(lg_g, lg_o)
    assert r < LOGIT_TOL, f"{where}: logits differ by {r:.2e}"
    if margin(lg_o) > LOGIT_TOL:
        assert int(np.argmax(lg_g)) == int(np.argmax(lg_o)), f"{where}: greedy token differs"
        return True
    return False


def row_trace(q, s, c, n: int, i: int, final: bool = True):
    """Row i of a batch trace (per site [n][k]) in single-pass order."""
    qs, ss = [], []
    off = 0
    for k, _ in site_lengths(c, 1, final):
        qs.append(q[off + i * k: off + (i + 1) * k])
        ss.append(s[(off + i * k) // 32: (off + (i + 1) * k) // 32])
        off += n * k
    return np.concatenate(qs), np.concatenate(ss)
