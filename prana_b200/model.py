"""The `prana-model` decode API (crates/prana-model/src/lib.rs:17-23) on B200.

`Model.load` reads a GGUF file into HBM (gguf.rs:338-460); `KvCache`, `forward`,
`prefill`, `forward_batch`, `generate` and `generate_speculative` keep the
reference's names and semantics over token ids (the tokenizer is not on the
decode path).  Host buffers cross the ABI; only token ids and, on request,
logits leave the device.
"""
from __future__ import annotations

import ctypes as C
import weakref
from dataclasses import dataclass

import numpy as np

from . import _ffi
from ._ffi import ModelConfig, call
from .kernels import context


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32).reshape(-1))


@dataclass
class Config:
    """checkpoint.rs:32-65 Config (the fields the decode path reads)."""

    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int
    head_dim: int
    rope_theta: float
    norm_eps: float
    rope_neox: bool
    has_bias: bool
    shared_classifier: bool
    weight_bytes: int

    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def q_dim(self) -> int:
        return self.n_heads * self.head_dim


def tp_unique_id() -> bytes:
    """NCCL unique id (128 bytes) that rank 0 shares with every tensor-parallel rank."""
    buf = C.create_string_buffer(128)
    call("prana_tp_unique_id", buf)
    return buf.raw


PRECISION_F32, PRECISION_Q8 = 0, 1


class Model:
    def __init__(self, handle: C.c_void_p, device: int):
        self._h = handle
        self.device = device
        self._caches: "weakref.WeakSet[KvCache]" = weakref.WeakSet()
        c = ModelConfig()
        call("prana_model_config_get", handle, C.byref(c))
        self.config = Config(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, c.seq_len,
                             c.head_dim, c.rope_theta, c.norm_eps, bool(c.rope_neox), bool(c.has_bias),
                             bool(c.shared_classifier), c.weight_bytes)
        world, rank, peer = C.c_int(), C.c_int(), C.c_int()
        call("prana_model_tp_get", handle, C.byref(world), C.byref(rank), C.byref(peer))
        self.world, self.rank = world.value, rank.value
        self.peer_exchange = bool(peer.value)

    @classmethod
    def load(cls, path: str, device: int = 0, tp: "tuple[int, int, bytes] | None" = None,
             precision: int = PRECISION_F32) -> "Model":
        """Load a GGUF model (gguf::load, gguf.rs:338-460); tp = (world, rank,
        unique_id) loads this rank's tensor-parallel shard (every rank then calls
        the same model methods in the same order).  precision PRECISION_Q8 is
        the reference's `--q8`: dense tensors become quantize_q8 of them."""
        h = C.c_void_p()
        if precision != PRECISION_F32:
            if tp is not None and tp[0] != 1:
                raise ValueError("tensor parallelism loads at F32 precision")
            call("prana_model_load_gguf_ex", context(device), str(path).encode(), precision, C.byref(h))
        elif tp is None or tp[0] == 1:
            call("prana_model_load_gguf", context(device), str(path).encode(), C.byref(h))
        else:
            world, rank, uid = tp
            buf = C.create_string_buffer(bytes(uid), 128)
            call("prana_model_load_gguf_tp", context(device), str(path).encode(), world, rank, buf, C.byref(h))
        return cls(h, device)

    def local_kv_dim(self) -> int:
        """Width of this rank's KV-cache rows (its kv heads)."""
        return self.config.n_kv_heads // self.world * self.config.head_dim

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def stream(self) -> int:
        """cudaStream_t (as int) all model-level work runs on."""
        s = C.c_void_p()
        call("prana_ctx_stream", context(self.device), C.byref(s))
        return s.value or 0

    def close(self):
        """Free the model and every KV cache still attached to it."""
        for cache in list(getattr(self, "_caches", ())):
            cache.close()
        if getattr(self, "_h", None) is not None and self._h.value:
            _ffi.lib().prana_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KvCache:
    """KvCache::with_len (infer.rs:37-45): f16 K/V rows in HBM."""

    def __init__(self, model: Model, positions: int | None = None):
        self.model = model
        self.positions = min(positions or model.config.seq_len, model.config.seq_len)
        self._h = C.c_void_p()
        call("prana_kv_create", model.handle, self.positions, C.byref(self._h))
        model._caches.add(self)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def read(self, layer: int, is_v: bool, rows: int, first: int = 0) -> np.ndarray:
        """f16 bits of rows [first, first + rows) of one layer's K or V cache."""
        out = np.empty((rows, self.model.local_kv_dim()), dtype=np.uint16)
        call("prana_kv_read_rows", self._h, layer, int(is_v), first, rows, out.ctypes.data_as(C.c_void_p))
        return out

    def write(self, layer: int, is_v: bool, rows: np.ndarray) -> None:
        rows = np.ascontiguousarray(rows, dtype=np.uint16)
        call("prana_kv_write", self._h, layer, int(is_v), rows.shape[0], rows.ctypes.data_as(C.c_void_p))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _ffi.lib().prana_kv_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def forward(model: Model, cache: KvCache, token: int, pos: int, want_logits: bool = True):
    """forward (infer.rs:134-136): returns (logits or None, argmax token)."""
    logits = np.empty(model.config.vocab_size, dtype=np.float32) if want_logits else None
    nxt = C.c_uint32()
    call("prana_forward", model.handle, cache.handle, token, pos,
         logits.ctypes.data_as(C.c_void_p) if logits is not None else None, C.byref(nxt))
    return logits, nxt.value


def forward_trace(model: Model, cache: KvCache, token: int, pos: int):
    """Diagnostic forward: (logits, int8 activation rows, their scales) in CPU-path order."""
    c = model.config
    n = c.n_layers * (2 * c.dim + c.q_dim() + c.hidden_dim) + c.dim
    q = np.empty(n, np.int8)
    s = np.empty(n // 32, np.float32)
    logits = np.empty(c.vocab_size, np.float32)
    got = C.c_size_t()
    call("prana_forward_trace", model.handle, cache.handle, token, pos, logits.ctypes.data_as(C.c_void_p),
         q.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p), n, C.byref(got))
    assert got.value == n
    return logits, q, s


def batch_trace(model: Model, cache: KvCache, tokens, pos0: int, prefill: bool):
    """Diagnostic prefill (positions 0..n) or forward_batch (positions pos0..):
    (logits [n, vocab] or None, int8 activation rows, their scales); per layer
    the n rows of each site, then the final-norm rows (forward_batch only)."""
    c = model.config
    t = _u32(tokens)
    n = t.size
    total = n * (c.n_layers * (2 * c.dim + c.q_dim() + c.hidden_dim) + (0 if prefill else c.dim))
    q = np.empty(total, np.int8)
    s = np.empty(total // 32, np.float32)
    logits = None if prefill else np.empty((n, c.vocab_size), np.float32)
    got = C.c_size_t()
    call("prana_forward_batch_trace", model.handle, cache.handle, t.ctypes.data_as(C.c_void_p), n, pos0,
         int(prefill), logits.ctypes.data_as(C.c_void_p) if logits is not None else None,
         q.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p), total, C.byref(got))
    assert got.value == total
    return logits, q, s


def prefill(model: Model, cache: KvCache, tokens) -> None:
    """prefill (infer.rs:220-286)."""
    t = _u32(tokens)
    call("prana_prefill", model.handle, cache.handle, t.ctypes.data_as(C.c_void_p), t.size)


def forward_batch(model: Model, cache: KvCache, tokens, pos0: int, want_logits: bool = True):
    """forward_batch (infer.rs:296-374): returns (logits [n, vocab] or None, argmax per row)."""
    t = _u32(tokens)
    n = t.size
    logits = np.empty((n, model.config.vocab_size), dtype=np.float32) if want_logits else None
    am = np.empty(n, dtype=np.uint32)
    call("prana_forward_batch", model.handle, cache.handle, t.ctypes.data_as(C.c_void_p), n, pos0,
         logits.ctypes.data_as(C.c_void_p) if logits is not None else None, am.ctypes.data_as(C.c_void_p))
    return logits, am


def forward_multi(model: Model, caches, tokens, positions, want_logits: bool = True):
    """One token for each of len(caches) independent sequences (row i: tokens[i]
    at positions[i] over caches[i]); returns (logits [n, vocab] or None, argmax [n]).
    The reference's equivalent is one forward (infer.rs:142-211) per sequence."""
    t = _u32(tokens)
    n = t.size
    assert len(caches) == n and len(positions) == n
    handles = (C.c_void_p * n)(*[c.handle.value for c in caches])
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    logits = np.empty((n, model.config.vocab_size), dtype=np.float32) if want_logits else None
    am = np.empty(n, dtype=np.uint32)
    call("prana_forward_multi", model.handle, handles, n, t.ctypes.data_as(C.c_void_p), pos.ctypes.data_as(C.c_void_p),
         logits.ctypes.data_as(C.c_void_p) if logits is not None else None, am.ctypes.data_as(C.c_void_p))
    return logits, am


def forward_multi_trace(model: Model, caches, tokens, positions):
    """Diagnostic forward_multi: (logits [n, vocab], int8 activation rows, scales)
    in the batch-trace layout (per layer the n rows of each site, then the n
    final-norm rows)."""
    c = model.config
    t = _u32(tokens)
    n = t.size
    assert len(caches) == n and len(positions) == n
    handles = (C.c_void_p * n)(*[k.handle.value for k in caches])
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    total = n * (c.n_layers * (2 * c.dim + c.q_dim() + c.hidden_dim) + c.dim)
    q = np.empty(total, np.int8)
    s = np.empty(total // 32, np.float32)
    logits = np.empty((n, c.vocab_size), np.float32)
    got = C.c_size_t()
    call("prana_forward_multi_trace", model.handle, handles, n, t.ctypes.data_as(C.c_void_p),
         pos.ctypes.data_as(C.c_void_p), logits.ctypes.data_as(C.c_void_p), q.ctypes.data_as(C.c_void_p),
         s.ctypes.data_as(C.c_void_p), total, C.byref(got))
    assert got.value == total
    return logits, q, s


def generate(model: Model, prompt, steps: int, stop_id: int = -1) -> np.ndarray:
    """generate (infer.rs:696-771), greedy, over token ids."""
    p = _u32(prompt)
    out = np.empty(max(steps, 1), dtype=np.uint32)
    n = C.c_size_t()
    call("prana_generate", model.handle, p.ctypes.data_as(C.c_void_p), p.size, steps, stop_id,
         out.ctypes.data_as(C.c_void_p), C.byref(n))
    return out[: n.value].copy()


def forward_sampled(model: Model, cache: KvCache, token: int, pos: int, sampler) -> int:
    """forward_impl (infer.rs:142-211) followed by Sampler::sample on the device
    over the step's logits; returns the next id (the sampler moves past its draw)."""
    out = C.c_uint32()
    call("prana_forward_sampled", model.handle, cache.handle, token, pos, sampler.handle, C.byref(out))
    return out.value


def generate_sampled(model: Model, prompt, steps: int, sampler, stop_id: int = -1) -> np.ndarray:
    """generate (infer.rs:696-771) with a Sampler (prana_b200.sampler.Sampler):
    each sampled position draws on the device; the sampler is left where the
    reference's loop leaves it."""
    p = _u32(prompt)
    out = np.empty(max(steps, 1), dtype=np.uint32)
    n = C.c_size_t()
    call("prana_generate_sampled", model.handle, p.ctypes.data_as(C.c_void_p), p.size, steps, stop_id,
         sampler.handle, out.ctypes.data_as(C.c_void_p), C.byref(n))
    return out[: n.value].copy()


def generate_speculative(target: Model, draft: Model, prompt, steps: int, k: int, stop_id: int = -1):
    """generate_speculative (infer.rs:581-690): returns (ids, (proposed, accepted))."""
    p = _u32(prompt)
    out = np.empty(max(steps, 1), dtype=np.uint32)
    n = C.c_size_t()
    stats = (C.c_size_t * 2)()
    call("prana_generate_speculative", target.handle, draft.handle, p.ctypes.data_as(C.c_void_p), p.size, steps, k,
         stop_id, out.ctypes.data_as(C.c_void_p), C.byref(n), stats)
    return out[: n.value].copy(), (stats[0], stats[1])


class DecodeLoop:
    """Device-resident decode: the per-token graph replays back to back with
    the next id (greedy, or drawn by a sampler on the device) fed back on the
    device."""

    def __init__(self, model: Model, cache: KvCache):
        self.model, self.cache = model, cache

    def begin(self, token: int, pos: int, sampler=None) -> None:
        if sampler is None:
            call("prana_decode_begin", self.model.handle, self.cache.handle, token, pos)
        else:
            call("prana_decode_begin_sampled", self.model.handle, self.cache.handle, token, pos, sampler.handle)

    def run(self, n_steps: int) -> None:
        call("prana_decode_run", self.model.handle, self.cache.handle, n_steps)

    def tokens(self, max_n: int) -> np.ndarray:
        out = np.empty(max(max_n, 1), dtype=np.uint32)
        n = C.c_size_t()
        call("prana_decode_tokens", self.model.handle, self.cache.handle, out.ctypes.data_as(C.c_void_p), max_n, C.byref(n))
        return out[: n.value].copy()
