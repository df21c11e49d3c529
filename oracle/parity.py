"""Parity checks of the GPU model path against the CPU oracle (TEST
INFRASTRUCTURE, not product code: used by tests/ and by bench.py's CPU leg,
outside every timed region).

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
# The attention output is the one site whose f32 values differ by more than
# summation order over a few products: it sums softmax-weighted f16 rows over
# up to thousands of positions with the GPU's expf and another order (the
# attention kernels are held to 2e-5 normwise).  Its scales may differ by
# ATT_SCALE_TOL and its flips lie within ATT_TIE_TOL of a rounding boundary
# (127 x the value difference, with margin).
ATT_SCALE_TOL = 1e-4
ATT_TIE_TOL = 1e-2
# A GPU f16 K/V value must be the rounding of a value within this fraction of
# its row's largest magnitude of the oracle's f32 value (the f32 values come
# from sums whose order differs; their error scales with the terms, not with
# the possibly small result).
KV_TIE_TOL = 1e-5


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
        self.kv_flips = 0
        self.kv_total = 0

    def check(self, q_g, s_g, q_o, s_o, v_o, where: str, scale_tol: float = SCALE_TOL,
              tie_tol: float = TIE_TOL) -> None:
        """Every element of the GPU's rows equals the oracle's, or differs by one
        step at a rounding tie of the oracle's own value; scales agree."""
        q_g = np.asarray(q_g)
        q_o = np.asarray(q_o)
        assert q_g.shape == q_o.shape
        srel = float(np.max(np.abs(np.asarray(s_g, np.float64) - s_o) / np.maximum(np.abs(s_o), 1e-30)))
        assert srel <= scale_tol, f"{where}: scales differ by {srel:.1e}"
        d = q_g.astype(np.int32) - q_o
        self.total += d.size
        if not np.any(d):
            return
        assert np.max(np.abs(d)) <= 1, f"{where}: int8 activations differ by more than one step"
        idx = np.nonzero(d)[0]
        t = np.asarray(v_o, np.float64)[idx] / np.repeat(np.asarray(s_o, np.float64), 32)[idx]
        tie = np.abs(np.abs(t - np.trunc(t)) - 0.5)
        assert np.all(tie < tie_tol), f"{where}: a flip away from a rounding tie ({tie.max():.2e})"
        self.flips += int(idx.size)

    def check_kv(self, kv_g, kv_o, kv_val, where: str, kv_dim: int) -> None:
        """f16 K/V rows written from the same int8 inputs: every GPU value is the
        f16 rounding of some value within KV_TIE_TOL x (its row's largest
        magnitude) of the oracle's f32 value -- one ulp apart at a rounding tie,
        or a few subnormal-range ulps for values near zero."""
        a, b = f16_key(kv_g), f16_key(kv_o)
        d = np.abs(a - b)
        self.kv_total += d.size
        if not np.any(d):
            return
        idx = np.nonzero(d)[0]
        vals = np.asarray(kv_val, np.float32)
        row_max = np.max(np.abs(vals.reshape(-1, kv_dim)), axis=1)
        tau = (KV_TIE_TOL * row_max[idx // kv_dim]).astype(np.float32)
        x = vals[idx]
        lo = f16_key((x - tau).astype(np.float16).view(np.uint16))
        hi = f16_key((x + tau).astype(np.float16).view(np.uint16))
        ok = (a[idx] >= lo) & (a[idx] <= hi)
        assert np.all(ok), (f"{where}: {int((~ok).sum())} f16 K/V values are not roundings of the oracle's "
                            f"value within {KV_TIE_TOL:g} of the row (max {int(d.max())} ulps)")
        self.kv_flips += int(idx.size)

    def bounded(self, frac: float = 0.01, floor: int = 32) -> bool:
        return (self.flips <= max(floor, int(self.total * frac))
                and self.kv_flips <= max(floor, int(self.kv_total * frac)))


def f16_key(bits):
    """f16 bit patterns on one ordered integer line (+0 and -0 both 0)."""
    b = np.asarray(bits).astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def check_trace(c, q_g, s_g, q_o, s_o, v_o, flips: Flips, where: str, rows: int = 1, final: bool = True):
    off = 0
    for i, (k, r) in enumerate(site_lengths(c, rows, final)):
        n = k * r
        att = i % 4 == 1 and i < 4 * c.n_layers
        flips.check(q_g[off:off + n], s_g[off // 32:(off + n) // 32], q_o[off:off + n],
                    s_o[off // 32:(off + n) // 32], v_o[off:off + n], f"{where} site {i}",
                    ATT_SCALE_TOL if att else SCALE_TOL, ATT_TIE_TOL if att else TIE_TOL)
        off += n
    assert off == len(q_g)


def gpu_kv_rows(gkv, n_layers: int, first: int, n: int) -> np.ndarray:
    """The GPU cache's rows [first, first + n) of every layer: K rows, then V rows."""
    out = []
    for layer in range(n_layers):
        for is_v in (False, True):
            out.append(gkv.read(layer, is_v, n, first).reshape(-1))
    return np.concatenate(out)


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


def forced_decode(om, okv, gm, gkv, tok: int, pos: int, flips: Flips, where: str):
    """One decode step on both sides: the GPU's traced pass, then the oracle
    forced with its int8 rows and its f16 K/V row, every difference checked.
    Returns (GPU logits, oracle logits)."""
    from prana_b200 import model as pm

    c = gm.config
    lg_g, q_g, s_g = pm.forward_trace(gm, gkv, tok, pos)
    kv_g = gpu_kv_rows(gkv, c.n_layers, pos, 1)
    lg_o, q_o, s_o, v_o, kv_o, kv_v = om.forward_trace(okv, tok, pos, with_values=True, force=(q_g, s_g),
                                                        force_kv=kv_g)
    flips.check_kv(kv_g, kv_o, kv_v, where, c.n_kv_heads * c.head_dim)
    check_trace(c, q_g, s_g, q_o, s_o, v_o, flips, where)
    return lg_g, lg_o


def forced_batch(om, okv, gm, gkv, tokens, pos0: int, prefill: bool, flips: Flips, where: str):
    """prefill (positions 0..n) or forward_batch (positions pos0..) on both
    sides, the oracle forced as in forced_decode.  Returns (GPU logits, oracle
    logits), None for prefill."""
    from prana_b200 import model as pm

    c = gm.config
    n = len(tokens)
    first = 0 if prefill else pos0
    lg_g, q_g, s_g = pm.batch_trace(gm, gkv, tokens, pos0, prefill=prefill)
    kv_g = gpu_kv_rows(gkv, c.n_layers, first, n)
    lg_o, q_o, s_o, v_o, kv_o, kv_v = om.batch_trace(okv, tokens, pos0, verify=not prefill, with_values=True,
                                                      force=(q_g, s_g), force_kv=kv_g)
    flips.check_kv(kv_g, kv_o, kv_v, where, c.n_kv_heads * c.head_dim)
    check_trace(c, q_g, s_g, q_o, s_o, v_o, flips, where, rows=n, final=not prefill)
    return lg_g, lg_o


# ---- temperature sampling (sampler.rs:22-37) ----
# The reference subtracts the f32 probabilities from the draw r one at a time
# after summing the exps sequentially in f32; the device sums in f64.  Where
# the two pick different ids, r must lie at every bucket boundary k between
# them within what the reference's own arithmetic moves that boundary:
#   - its running value r_k versus r - C(k) exactly (measured here), and
#   - its sequential f32 sum of the exps, which scales every probability by
#     sum(p) - 1 (measured here), plus 1e-6 relative for CUDA's expf (2 ulp)
#     and the device's f64 sum rounded once to f32.
SAMPLE_REL_TOL = 1e-6


def sample_boundary_gap(probs, r: float, a: int, b: int, tol: float | None = None) -> float:
    """Largest excess over the allowed distance of |r - C(k)| for k in [a, b),
    where C is the exact cumulative of the oracle's f32 probabilities; <= 0
    means every boundary between ids a and b is within tolerance of r.  tol
    (absolute) replaces the softmax terms when the logits themselves differ."""
    p = np.asarray(probs, np.float32)
    scale_err = abs(float(np.sum(p, dtype=np.float64)) - 1.0) + SAMPLE_REL_TOL
    run = np.float32(r)
    worst = -np.inf
    exact = 0.0
    for k in range(b):
        run = np.float32(run - p[k])  # the reference's running value, f32
        exact += float(p[k])
        if k >= a:
            seq_err = abs((float(r) - exact) - float(run))
            allowed = seq_err + (tol if tol is not None else scale_err * exact + 1e-9)
            worst = max(worst, abs(float(r) - exact) - allowed)
    return worst
