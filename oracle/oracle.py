"""ctypes binding of the oracle (TEST INFRASTRUCTURE, not product code).

The oracle is the C restatement of Prana's CPU decode path in this folder.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
as the checker / the timed CPU baseline, never as the thing measured.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

TIER_AUTO, TIER_SCALAR, TIER_AVX2, TIER_VNNI = 0, 1, 2, 3

P = C.c_void_p
SZ = C.c_size_t


class Config(C.Structure):
    _fields_ = [("dim", SZ), ("hidden_dim", SZ), ("n_layers", SZ), ("n_heads", SZ), ("n_kv_heads", SZ),
                ("vocab_size", SZ), ("seq_len", SZ), ("head_dim", SZ), ("rope_theta", C.c_float),
                ("norm_eps", C.c_float), ("rope_neox", C.c_int), ("has_bias", C.c_int),
                ("shared_classifier", C.c_int)]


class Matrix(C.Structure):
    _fields_ = [("kind", C.c_int), ("rows", SZ), ("cols", SZ), ("f32", P), ("q", P), ("scales", P), ("blocks", P)]


_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sig = {
            "or_f16_to_f32": ([C.c_uint16], C.c_float),
            "or_f32_to_f16": ([C.c_float], C.c_uint16),
            "or_quantize_acts": ([P, SZ, P, P, P], None),
            "or_quantize_q8": ([SZ, SZ, P, P, P], None),
            "or_dequant_q40_block": ([P, P], None),
            "or_q4k_scale_min": ([C.c_int, P, P, P], None),
            "or_dequant_q4k_block": ([P, P], None),
            "or_dequant_q6k_block": ([P, P], None),
            "or_dot_q8_q8": ([C.c_int, P, P, SZ, P, P], C.c_float),
            "or_dot_q40_q8": ([C.c_int, P, P, P, SZ, P, P], C.c_float),
            "or_dot_q4k_q8": ([C.c_int, P, P, P, SZ, P, P], C.c_float),
            "or_dot_q6k_q8": ([P, P, SZ, P, P], C.c_float),
            "or_dot_f32": ([C.c_int, P, P, SZ], C.c_float),
            "or_block_dots": ([C.c_int, P, SZ, P, P], None),
            "or_simd_available": ([], C.c_int),
            "or_vnni_available": ([], C.c_int),
            "or_default_tier": ([], C.c_int),
            "or_pool_threads": ([], C.c_int),
            "or_pool_set_threads": ([C.c_int], None),
            "or_matrix_from_gguf": ([P, C.c_int, SZ, SZ, P], C.c_int),
            "or_matrix_free": ([P], None),
            "or_matrix_dequant": ([P, P], None),
            "or_matmul": ([C.c_int, P, P, SZ, P], None),
            "or_matmul_prefill": ([C.c_int, P, P, P, P, SZ, P], None),
            "or_rmsnorm": ([P, P, SZ, SZ, C.c_float, P], None),
            "or_silu": ([P, SZ], None),
            "or_softmax": ([P, SZ, P], None),
            "or_rope_interleaved": ([P, SZ, SZ, SZ, C.c_float], None),
            "or_rope_neox": ([P, SZ, SZ, SZ, C.c_float], None),
            "or_rope_batch": ([P, SZ, SZ, SZ, C.c_float], None),
            "or_rope_table": ([SZ, SZ, C.c_float, C.c_int, P, P], None),
            "or_f16_kv_write": ([P, SZ, SZ, P, SZ], None),
            "or_attention_decode": ([P, P, P, SZ, SZ, SZ, SZ, P], None),
            "or_attention_verify": ([P, P, P, SZ, SZ, SZ, SZ, SZ, P], None),
            "or_attention": ([P, P, P, SZ, SZ, SZ, SZ, P], None),
            "or_argmax": ([P, SZ], C.c_uint32),
            "or_xorshift_next": ([P], C.c_uint64),
            "or_xorshift_f32": ([P], C.c_float),
            "or_sample": ([P, SZ, C.c_float, P, P, P], C.c_uint32),
            "or_generate_sampled": ([P, P, SZ, SZ, C.c_int64, C.c_float, P, P], SZ),
            "or_model_load": ([C.c_char_p, C.c_int, C.c_char_p, SZ], P),
            "or_model_load_ex": ([C.c_char_p, C.c_int, C.c_int, C.c_char_p, SZ], P),
            "or_model_free": ([P], None),
            "or_model_config": ([P, C.POINTER(Config)], None),
            "or_model_matrix": ([P, C.c_int, C.c_char_p], P),
            "or_kv_create": ([P, SZ], P),
            "or_kv_free": ([P], None),
            "or_kv_layer": ([P, C.c_int, C.c_int], P),
            "or_forward": ([P, P, C.c_uint32, SZ, P], None),
            "or_forward_trace": ([P, P, C.c_uint32, SZ, P, P, P, P, SZ], SZ),
            "or_forward_trace_forced": ([P, P, C.c_uint32, SZ, P, P, P, P, SZ, P, P, P, P, P, SZ], SZ),
            "or_batch_trace": ([P, P, P, SZ, SZ, C.c_int, P, P, P, P, SZ, P, P, P, P, P, SZ], SZ),
            "or_prefill": ([P, P, P, SZ], None),
            "or_forward_batch": ([P, P, P, SZ, SZ, P], None),
            "or_generate": ([P, P, SZ, SZ, C.c_int64, P], SZ),
            "or_generate_speculative": ([P, P, P, SZ, SZ, SZ, C.c_int64, P, P], SZ),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def ptr(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def quantize_acts(a: np.ndarray):
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    k = a.size
    q = np.empty(k, np.int8)
    s = np.empty(k // 32, np.float32)
    sm = np.empty(k // 32, np.int32)
    lib().or_quantize_acts(ptr(a), k, ptr(q), ptr(s), ptr(sm))
    return q, s, sm


def quantize_acts_rows(a: np.ndarray):
    rows = [quantize_acts(r) for r in np.asarray(a, np.float32).reshape(-1, a.shape[-1])]
    return (np.stack([r[0] for r in rows]), np.stack([r[1] for r in rows]), np.stack([r[2] for r in rows]))


class OSampler:
    """Sampler (sampler.rs:6-37): greedy when temperature <= 0, else temperature
    sampling over the xorshift64* stream seeded with seed (0 reads as 1)."""

    def __init__(self, temperature: float, seed: int):
        self.temperature = float(temperature)
        self.state = np.array([max(int(seed), 1)], np.uint64)

    def next_f32(self) -> float:
        return float(lib().or_xorshift_f32(ptr(self.state)))

    def sample(self, logits: np.ndarray):
        """(token, softmax probabilities or None, draw r or None)"""
        lg = np.ascontiguousarray(logits, np.float32)
        greedy = self.temperature <= 0.0
        probs = None if greedy else np.empty(lg.size, np.float32)
        r = np.zeros(1, np.float32)
        tok = lib().or_sample(ptr(lg), lg.size, self.temperature, ptr(self.state),
                              None if greedy else ptr(probs), ptr(r))
        return int(tok), probs, (None if greedy else float(r[0]))


class OMatrix:
    """An oracle weight matrix built from GGUF block bytes (gguf.rs:271-305)."""

    def __init__(self, ggml_type: int, rows: int, cols: int, raw: np.ndarray):
        self._raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        self.m = Matrix()
        if lib().or_matrix_from_gguf(C.byref(self.m), ggml_type, rows, cols, ptr(self._raw)):
            raise ValueError("oracle: bad matrix")
        self.rows, self.cols = rows, cols

    def dequant(self) -> np.ndarray:
        out = np.empty((self.rows, self.cols), np.float32)
        lib().or_matrix_dequant(C.byref(self.m), ptr(out))
        return out

    def matmul(self, a: np.ndarray, tier: int = TIER_AUTO) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        n = a.size // self.cols
        out = np.empty((n, self.rows), np.float32)
        lib().or_matmul(tier, C.byref(self.m), ptr(a), n, ptr(out))
        return out

    def matmul_prefill(self, q, s, sm, tier: int = TIER_AUTO) -> np.ndarray:
        q, s, sm = (np.ascontiguousarray(x) for x in (q, s, sm))
        n = q.shape[0]
        out = np.empty((n, self.rows), np.float32)
        lib().or_matmul_prefill(tier, C.byref(self.m), ptr(q), ptr(s), ptr(sm), n, ptr(out))
        return out

    def __del__(self):
        try:
            lib().or_matrix_free(C.byref(self.m))
        except Exception:
            pass


class OQ8Matrix(OMatrix):
    """The reference's in-memory QuantMatrix built by quantize_q8 (int8 plus f32
    scales, matmul.rs:21-30, 61-84), multiplied by the oracle's Q8 kernels."""

    def __init__(self, rows: int, cols: int, w: np.ndarray):
        w = np.ascontiguousarray(w, np.float32).reshape(-1)
        self._q = np.empty(rows * cols, np.int8)
        self._s = np.empty(rows * cols // 32, np.float32)
        lib().or_quantize_q8(rows, cols, ptr(w), ptr(self._q), ptr(self._s))
        self.m = Matrix()
        self.m.kind, self.m.rows, self.m.cols = 8, rows, cols
        self.m.q, self.m.scales = self._q.ctypes.data, self._s.ctypes.data
        self.rows, self.cols = rows, cols

    def __del__(self):  # the planes belong to numpy
        pass


def block_dots(ggml_type: int, aq: np.ndarray, row_bytes: np.ndarray, k: int) -> np.ndarray:
    n = k // 16 if ggml_type == 14 else k // 32
    out = np.zeros(n, np.int32)
    lib().or_block_dots(ggml_type, ptr(np.ascontiguousarray(aq)), k, ptr(np.ascontiguousarray(row_bytes)), ptr(out))
    return out


class OModel:
    def __init__(self, path: str, tier: int = TIER_AUTO, precision: int = 0):
        """gguf::load(path, precision): precision 0 = F32 (the default), 1 = Q8 (`--q8`)."""
        err = C.create_string_buffer(512)
        self.h = lib().or_model_load_ex(str(path).encode(), tier, precision, err, 512)
        if not self.h:
            raise ValueError("oracle load failed: " + err.value.decode())
        self.c = Config()
        lib().or_model_config(self.h, C.byref(self.c))

    def kv(self, positions: int):
        return OKv(self, positions)

    def forward(self, kv: "OKv", token: int, pos: int, want_logits: bool = True):
        lg = np.empty(self.c.vocab_size, np.float32) if want_logits else None
        lib().or_forward(self.h, kv.h, token, pos, ptr(lg) if lg is not None else None)
        return lg

    def trace_len(self) -> int:
        c = self.c
        return c.n_layers * (2 * c.dim + c.n_heads * c.head_dim + c.hidden_dim) + c.dim

    def kv_trace_len(self, rows: int = 1) -> int:
        return self.c.n_layers * 2 * rows * self.c.n_kv_heads * self.c.head_dim

    def forward_trace(self, kv: "OKv", token: int, pos: int, with_values: bool = False, force=None, force_kv=None):
        """(logits, int8 activation rows, scales[, the f32 values quantized]) in forward order.

        force = (q, scales) of another pass's trace: the oracle still records
        its own quantized rows, but every matmul takes the given rows instead.
        force_kv = f16 K/V rows of another pass (per layer: the K row, then the
        V row): the cache keeps those instead of this pass's own; the return
        value then ends with (own f16 rows, their f32 values).  Test
        instrumentation (or_forward_trace_forced)."""
        n = self.trace_len()
        q = np.empty(n, np.int8)
        s = np.empty(n // 32, np.float32)
        v = np.empty(n, np.float32) if with_values else None
        lg = np.empty(self.c.vocab_size, np.float32)
        if force is None and force_kv is None:
            got = lib().or_forward_trace(self.h, kv.h, token, pos, ptr(lg), ptr(q), ptr(s),
                                         ptr(v) if v is not None else None, n)
            assert got == n
            return (lg, q, s, v) if with_values else (lg, q, s)
        fq = fs = fkv = kv_own = kv_val = None
        if force is not None:
            fq = np.ascontiguousarray(force[0], np.int8)
            fs = np.ascontiguousarray(force[1], np.float32)
            assert fq.size == n and fs.size == n // 32
        nkv = self.kv_trace_len(1)
        if force_kv is not None:
            fkv = np.ascontiguousarray(force_kv, np.uint16).reshape(-1)
            assert fkv.size == nkv
            kv_own = np.empty(nkv, np.uint16)
            kv_val = np.empty(nkv, np.float32)
        got = lib().or_forward_trace_forced(self.h, kv.h, token, pos, ptr(lg), ptr(q), ptr(s),
                                            ptr(v) if v is not None else None, n,
                                            ptr(fq) if fq is not None else None, ptr(fs) if fs is not None else None,
                                            ptr(kv_own) if kv_own is not None else None,
                                            ptr(kv_val) if kv_val is not None else None,
                                            ptr(fkv) if fkv is not None else None, nkv)
        assert got == n
        out = (lg, q, s, v) if with_values else (lg, q, s)
        return out + (kv_own, kv_val) if force_kv is not None else out

    def batch_trace_len(self, n: int, verify: bool) -> int:
        c = self.c
        return n * (c.n_layers * (2 * c.dim + c.n_heads * c.head_dim + c.hidden_dim) + (c.dim if verify else 0))

    def batch_trace(self, kv: "OKv", tokens, pos0: int, verify: bool, with_values: bool = False, force=None,
                    force_kv=None):
        """prefill (verify False, positions 0..n) or forward_batch (verify True) with
        the activation trace: per layer the n rows of each site, then the
        final-norm rows (verify only).  Returns (logits [n, vocab] or None, q,
        scales[, values][, own K/V rows, their f32 values]); force and force_kv
        (per layer: n K rows, then n V rows) as in forward_trace."""
        t = np.ascontiguousarray(tokens, np.uint32)
        n = self.batch_trace_len(t.size, verify)
        q = np.empty(n, np.int8)
        s = np.empty(n // 32, np.float32)
        v = np.empty(n, np.float32) if with_values else None
        lg = np.empty((t.size, self.c.vocab_size), np.float32) if verify else None
        fq = fs = fkv = kv_own = kv_val = None
        if force is not None:
            fq = np.ascontiguousarray(force[0], np.int8)
            fs = np.ascontiguousarray(force[1], np.float32)
            assert fq.size == n and fs.size == n // 32
        nkv = self.kv_trace_len(t.size)
        if force_kv is not None:
            fkv = np.ascontiguousarray(force_kv, np.uint16).reshape(-1)
            assert fkv.size == nkv
            kv_own = np.empty(nkv, np.uint16)
            kv_val = np.empty(nkv, np.float32)
        got = lib().or_batch_trace(self.h, kv.h, ptr(t), t.size, pos0, int(verify),
                                   ptr(lg) if lg is not None else None, ptr(q), ptr(s),
                                   ptr(v) if v is not None else None, n,
                                   ptr(fq) if fq is not None else None, ptr(fs) if fs is not None else None,
                                   ptr(kv_own) if kv_own is not None else None,
                                   ptr(kv_val) if kv_val is not None else None,
                                   ptr(fkv) if fkv is not None else None, nkv)
        assert got == n
        out = (lg, q, s, v) if with_values else (lg, q, s)
        return out + (kv_own, kv_val) if force_kv is not None else out

    def prefill(self, kv: "OKv", tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        lib().or_prefill(self.h, kv.h, ptr(t), t.size)

    def forward_batch(self, kv: "OKv", tokens, pos0: int):
        t = np.ascontiguousarray(tokens, np.uint32)
        lg = np.empty((t.size, self.c.vocab_size), np.float32)
        lib().or_forward_batch(self.h, kv.h, ptr(t), t.size, pos0, ptr(lg))
        return lg

    def generate(self, prompt, steps: int, stop_id: int = -1) -> np.ndarray:
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max(steps, 1), np.uint32)
        n = lib().or_generate(self.h, ptr(p), p.size, steps, stop_id, ptr(out))
        return out[:n].copy()

    def generate_sampled(self, prompt, steps: int, temperature: float, seed: int, stop_id: int = -1):
        """generate with Sampler::new(temperature, seed); returns (tokens, xorshift state after the last draw)."""
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max(steps, 1), np.uint32)
        st = np.array([seed], np.uint64)
        n = lib().or_generate_sampled(self.h, ptr(p), p.size, steps, stop_id, temperature, ptr(st), ptr(out))
        return out[:n].copy(), int(st[0])

    def generate_speculative(self, draft: "OModel", prompt, steps: int, k: int, stop_id: int = -1):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max(steps, 1), np.uint32)
        stats = np.zeros(2, np.uint64)
        n = lib().or_generate_speculative(self.h, draft.h, ptr(p), p.size, steps, k, stop_id, ptr(out), ptr(stats))
        return out[:n].copy(), (int(stats[0]), int(stats[1]))

    def __del__(self):
        try:
            lib().or_model_free(self.h)
        except Exception:
            pass


class OKv:
    def __init__(self, m: OModel, positions: int):
        self.m = m
        self.h = lib().or_kv_create(m.h, positions)
        self.positions = min(positions, m.c.seq_len)

    def set_layer(self, l: int, is_v: bool, rows: np.ndarray) -> None:
        kv_dim = self.m.c.n_kv_heads * self.m.c.head_dim
        p = lib().or_kv_layer(self.h, l, int(is_v))
        dst = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint16)), shape=(self.positions, kv_dim))
        dst[: rows.shape[0]] = rows

    def layer(self, l: int, is_v: bool) -> np.ndarray:
        kv_dim = self.m.c.n_kv_heads * self.m.c.head_dim
        p = lib().or_kv_layer(self.h, l, int(is_v))
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint16)), shape=(self.positions, kv_dim)).copy()

    def __del__(self):
        try:
            lib().or_kv_free(self.h)
        except Exception:
            pass
