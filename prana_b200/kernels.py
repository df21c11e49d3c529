"""The `prana-kernels` function surface (crates/prana-kernels/src/lib.rs:35-54) on
B200, over torch CUDA tensors.

Each function keeps the reference's name, argument meaning and error
behaviour (shape violations raise, as the Rust asserts panic) and runs the
sm_100a kernels of libprana_cuda.so on the caller's current torch stream.
Device memory comes from torch; torch is plumbing here, the arithmetic is the
library's.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _ffi
from ._ffi import TYPE_F16, TYPE_F32, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, call

Q8_BLOCK = 32
QK_K = 256
BLOCK_BYTES = {TYPE_Q8_0: (32, 34), TYPE_Q4_0: (32, 18), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}

_ctxs: dict[int, C.c_void_p] = {}


def context(device: int | None = None) -> C.c_void_p:
    """The library context of a CUDA device, bound to torch's current stream."""
    if device is None:
        device = torch.cuda.current_device()
    ctx = _ctxs.get(device)
    if ctx is None:
        ctx = C.c_void_p()
        call("prana_ctx_create", device, C.byref(ctx))
        _ctxs[device] = ctx
    # torch reports its legacy default stream as handle 0; the ABI's NULL means
    # "the context's own stream", so pass cudaStreamLegacy (0x1) explicitly.
    handle = torch.cuda.current_stream(device).cuda_stream or 1
    call("prana_ctx_set_stream", ctx, C.c_void_p(handle))
    return ctx


def quantize_q8(rows: int, cols: int, w) -> tuple[np.ndarray, np.ndarray]:
    """quantize_q8 (matmul.rs:61-84) on the host: (int8 [rows, cols], f32 scales [rows, cols / 32])."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(rows, cols)
    q = np.empty((rows, cols), np.int8)
    s = np.empty((rows, cols // 32), np.float32)
    call("prana_quantize_q8", rows, cols, w.ctypes.data_as(C.c_void_p), q.ctypes.data_as(C.c_void_p),
         s.ctypes.data_as(C.c_void_p))
    return q, s


def synchronize(device: int | None = None) -> None:
    """Wait for this device's kernel-level calls; raises PranaError
    (PRANA_E_TIMEOUT) when a bounded device wait gave up in one of them."""
    call("prana_ctx_synchronize", context(device))


def debug_wait_timeout(which: int, polls: int, device: int | None = None) -> int:
    """Run one bounded device wait on data that never arrives (0: an mbarrier,
    1: the peer exchange's receive wait on local buffers) and return the status
    code the library reports (PRANA_E_TIMEOUT, -6, when the wait gave up)."""
    return int(_ffi.lib().prana_debug_wait_timeout(context(device), which, polls))


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


class QuantMatrix:
    """A [rows, cols] weight matrix resident in HBM in its repacked block format
    (QuantMatrix, matmul.rs:21-57, and KQuantMatrix, kquant.rs:116-233)."""

    def __init__(self, ggml_type: int, rows: int, cols: int, raw: bytes | np.ndarray, device: int | None = None):
        if ggml_type in BLOCK_BYTES:
            bv, bb = BLOCK_BYTES[ggml_type]
            if cols % bv:
                raise ValueError(f"cols must be a multiple of {bv}")
            need = rows * cols // bv * bb
        elif ggml_type == TYPE_F32:
            need = rows * cols * 4
        elif ggml_type == TYPE_F16:
            need = rows * cols * 2
        else:
            raise ValueError(f"unsupported ggml type {ggml_type}")
        buf = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray)) else raw.view(np.uint8).reshape(-1))
        if buf.size != need:
            raise ValueError(f"expected {need} bytes of packed blocks, got {buf.size}")
        self.ggml_type, self.rows, self.cols = ggml_type, rows, cols
        self.device = torch.cuda.current_device() if device is None else device
        self._h = C.c_void_p()
        call("prana_weight_upload", context(self.device), ggml_type, rows, cols, buf.ctypes.data_as(C.c_void_p), C.byref(self._h))

    @classmethod
    def quantize_q8(cls, rows: int, cols: int, w, device: int | None = None) -> "QuantMatrix":
        """Linear::new(w, Precision::Q8): quantize_q8 (matmul.rs:61-84) of a dense
        f32 [rows, cols] matrix, resident in HBM as int8 with f32 scales."""
        self = cls.__new__(cls)
        self.ggml_type, self.rows, self.cols = TYPE_Q8_0, rows, cols
        self.device = torch.cuda.current_device() if device is None else device
        self._h = C.c_void_p()
        f = np.ascontiguousarray(w, dtype=np.float32).reshape(rows, cols)
        call("prana_weight_upload_q8", context(self.device), rows, cols, f.ctypes.data_as(C.c_void_p),
             C.byref(self._h))
        return self

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def stored_bytes(self) -> int:
        n = C.c_size_t()
        call("prana_weight_bytes", self._h, C.byref(n))
        return n.value

    def __del__(self):
        try:
            h = getattr(self, "_h", None)
            if h is not None and h.value:
                _ffi.lib().prana_weight_free(h)
                self._h = None
        except Exception:  # interpreter shutdown: the library may already be gone
            pass


KQuantMatrix = QuantMatrix


class QuantActs:
    """Activation rows quantized per 32-group (matmul.rs:95-103)."""

    def __init__(self, q: torch.Tensor, scales: torch.Tensor, sums: torch.Tensor):
        self.q, self.scales, self.sums = q, scales, sums


def quantize_acts(a: torch.Tensor) -> QuantActs:
    """quantize_acts (matmul.rs:105-127) for each row of `a` ([rows, k] or [k])."""
    a2 = a.reshape(-1, a.shape[-1]) if a.dim() > 1 else a.reshape(1, -1)
    rows, k = a2.shape
    if k % Q8_BLOCK:
        raise ValueError("activation length must be a multiple of 32")
    q = torch.empty((rows, k), dtype=torch.int8, device=a.device)
    s = torch.empty((rows, k // 32), dtype=torch.float32, device=a.device)
    sm = torch.empty((rows, k // 32), dtype=torch.int32, device=a.device)
    call("prana_quantize_acts", context(a.device.index), _ptr(a2), rows, k, _ptr(q), _ptr(s), _ptr(sm))
    return QuantActs(q, s, sm)


def _out(n_tokens: int, rows: int, device) -> torch.Tensor:
    return torch.empty((n_tokens, rows), dtype=torch.float32, device=device)


def matmul_q8_f32(a: torch.Tensor, w: QuantMatrix, n_tokens: int) -> torch.Tensor:
    """matmul_q8_f32 (matmul.rs:162-178): [n_tokens, cols] f32 -> [n_tokens, rows]."""
    if a.numel() != n_tokens * w.cols:
        raise ValueError("a must hold n_tokens * cols values")
    out = _out(n_tokens, w.rows, a.device)
    call("prana_matmul_q8_f32", context(a.device.index), _ptr(a), w.handle, n_tokens, _ptr(out))
    return out


def matmul_kquant_f32(a: torch.Tensor, m: QuantMatrix, n_tokens: int) -> torch.Tensor:
    """matmul_kquant_f32 (kquant.rs:323-333)."""
    if a.numel() != n_tokens * m.cols:
        raise ValueError("a must hold n_tokens * cols values")
    out = _out(n_tokens, m.rows, a.device)
    call("prana_matmul_kquant_f32", context(a.device.index), _ptr(a), m.handle, n_tokens, _ptr(out))
    return out


def matmul_q8_prefill(acts: QuantActs, w: QuantMatrix) -> torch.Tensor:
    """matmul_q8_prefill (matmul.rs:185-187): already-quantized rows."""
    n = acts.q.shape[0]
    out = _out(n, w.rows, acts.q.device)
    call("prana_matmul_q8_prefill", context(acts.q.device.index), _ptr(acts.q), _ptr(acts.scales), _ptr(acts.sums), n, w.handle, _ptr(out))
    return out


def matmul_kquant_prefill(acts: QuantActs, m: QuantMatrix) -> torch.Tensor:
    """matmul_kquant_prefill (kquant.rs:368-370)."""
    n = acts.q.shape[0]
    out = _out(n, m.rows, acts.q.device)
    call("prana_matmul_kquant_prefill", context(acts.q.device.index), _ptr(acts.q), _ptr(acts.scales), _ptr(acts.sums), n, m.handle, _ptr(out))
    return out


def qgemm(acts: QuantActs, w: QuantMatrix) -> torch.Tensor:
    """The quantized rows times `w` on the tensor cores (tcgen05, one MMA per
    block): the products of matmul_q8_prefill / matmul_kquant_prefill."""
    n = acts.q.shape[0]
    out = _out(n, w.rows, acts.q.device)
    call("prana_qgemm", context(acts.q.device.index), _ptr(acts.q), _ptr(acts.scales), _ptr(acts.sums), n, w.handle,
         _ptr(out))
    return out


def qgemm_block_dots(acts: QuantActs, w: QuantMatrix) -> torch.Tensor:
    """Per-block int32 dots the tensor cores produce: [n_tokens, rows, blocks]
    (blocks = cols / 32, or cols / 16 for Q6_K)."""
    n = acts.q.shape[0]
    nb = w.cols // 16 if w.ggml_type == TYPE_Q6_K else w.cols // 32
    out = torch.zeros((n, w.rows, nb), dtype=torch.int32, device=acts.q.device)
    call("prana_qgemm_block_dots", context(acts.q.device.index), _ptr(acts.q), _ptr(acts.scales), _ptr(acts.sums), n,
         w.handle, _ptr(out))
    return out


def matmul_f32(a: torch.Tensor, w: QuantMatrix, n_tokens: int) -> torch.Tensor:
    """matmul_f32 (matmul.rs:150-156) over an F32 weight."""
    out = _out(n_tokens, w.rows, a.device)
    call("prana_matmul_f32", context(a.device.index), _ptr(a), w.handle, n_tokens, _ptr(out))
    return out


def block_dots(w: QuantMatrix, row: int, acts: QuantActs) -> torch.Tensor:
    """Per-block int32 dots of weight row `row` against activation row 0 of `acts`
    (the bit-exact quantities of the reference's scalar dots)."""
    n = w.cols // 16 if w.ggml_type == TYPE_Q6_K else w.cols // 32
    out = torch.zeros(n, dtype=torch.int32, device=acts.q.device)
    call("prana_block_dots", context(acts.q.device.index), w.handle, row, _ptr(acts.q), _ptr(acts.sums), _ptr(out))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, rows: int, dim: int, eps: float) -> torch.Tensor:
    """rmsnorm (norms.rs:9-23)."""
    if x.numel() != rows * dim or weight.numel() != dim:
        raise ValueError("shape mismatch")
    out = torch.empty_like(x)
    call("prana_rmsnorm", context(x.device.index), _ptr(x), _ptr(weight), rows, dim, C.c_float(eps), _ptr(out))
    return out


def silu(x: torch.Tensor) -> None:
    """silu in place (norms.rs:27-31)."""
    call("prana_silu", context(x.device.index), _ptr(x), x.numel())


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> None:
    """gate = silu(gate) * up in place (infer.rs:193-199)."""
    call("prana_silu_mul", context(gate.device.index), _ptr(gate), _ptr(up), gate.numel())


def softmax(logits: torch.Tensor) -> torch.Tensor:
    """softmax (norms.rs:44-56) over the last dimension."""
    x2 = logits.reshape(-1, logits.shape[-1]) if logits.numel() else logits
    out = torch.empty_like(logits)
    if logits.numel():
        call("prana_softmax", context(logits.device.index), _ptr(x2), x2.shape[0], x2.shape[1], _ptr(out))
    return out


def rope_interleaved(x: torch.Tensor, pos: int, head_dim: int, theta_base: float) -> None:
    """rope_interleaved (attention.rs:90-101) in place; rows of a 2-D x sit at pos, pos+1, ..."""
    rows = x.shape[0] if x.dim() == 2 else 1
    call("prana_rope_interleaved", context(x.device.index), _ptr(x), rows, x.shape[-1], pos, head_dim, C.c_float(theta_base))


def rope_neox(x: torch.Tensor, pos: int, head_dim: int, theta_base: float) -> None:
    """rope_neox (attention.rs:107-121) in place."""
    rows = x.shape[0] if x.dim() == 2 else 1
    call("prana_rope_neox", context(x.device.index), _ptr(x), rows, x.shape[-1], pos, head_dim, C.c_float(theta_base))


def f16_kv_write(cache: torch.Tensor, first_row: int, kv_stride: int, src: torch.Tensor) -> None:
    """f16_kv_write (attention.rs:47-52): cache holds f16 bits (int16/float16 storage)."""
    if (first_row * kv_stride + src.numel()) > cache.numel():
        raise ValueError("write past the end of the cache")
    call("prana_f16_kv_write", context(src.device.index), _ptr(cache), first_row, kv_stride, _ptr(src), src.numel())


def attention_decode(q, k_cache, v_cache, pos, n_heads, n_kv_heads, head_dim) -> torch.Tensor:
    """attention_decode (attention.rs:129-160) over an f16 cache [capacity, n_kv*hd]."""
    if n_kv_heads <= 0 or n_heads % n_kv_heads:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    if k_cache.numel() < (pos + 1) * n_kv_heads * head_dim:
        raise ValueError("k_cache not filled to pos")
    out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    call("prana_attention_decode", context(q.device.index), _ptr(q), _ptr(k_cache), _ptr(v_cache), pos, n_heads, n_kv_heads, head_dim, _ptr(out))
    return out


def attention_decode_noalloc(q, k_cache, v_cache, pos, n_heads, n_kv_heads, head_dim, out=None) -> torch.Tensor:
    """attention_decode on the library's static split scratch: the call itself
    allocates no device memory (pass `out` to avoid the output allocation too).
    Calls that overlap in time share that scratch and must be serialized."""
    if n_kv_heads <= 0 or n_heads % n_kv_heads:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    if k_cache.numel() < (pos + 1) * n_kv_heads * head_dim:
        raise ValueError("k_cache not filled to pos")
    if out is None:
        out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    call("prana_attention_decode_noalloc", context(q.device.index), _ptr(q), _ptr(k_cache), _ptr(v_cache), pos,
         n_heads, n_kv_heads, head_dim, _ptr(out))
    return out


def attention_verify(q, k_cache, v_cache, pos0, seq, n_heads, n_kv_heads, head_dim) -> torch.Tensor:
    """attention_verify (attention.rs:296-333): seq query rows at pos0.."""
    if k_cache.numel() < (pos0 + seq) * n_kv_heads * head_dim:
        raise ValueError("cache not filled to pos0+seq")
    out = torch.empty((seq, n_heads * head_dim), dtype=torch.float32, device=q.device)
    call("prana_attention_verify", context(q.device.index), _ptr(q), _ptr(k_cache), _ptr(v_cache), pos0, seq, n_heads, n_kv_heads, head_dim, _ptr(out))
    return out


def attention(q, k, v, seq, n_heads, n_kv_heads, head_dim) -> torch.Tensor:
    """attention (attention.rs:236-284): causal over f32 in-window K/V."""
    if n_kv_heads <= 0 or n_heads % n_kv_heads:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    out = torch.empty((seq, n_heads * head_dim), dtype=torch.float32, device=q.device)
    call("prana_attention", context(q.device.index), _ptr(q), _ptr(k), _ptr(v), seq, n_heads, n_kv_heads, head_dim, _ptr(out))
    return out


def argmax(logits: torch.Tensor) -> torch.Tensor:
    """First index of the maximum of each row (infer.rs:560-568)."""
    x2 = logits.reshape(-1, logits.shape[-1])
    out = torch.empty(x2.shape[0], dtype=torch.int32, device=logits.device)
    call("prana_argmax", context(logits.device.index), _ptr(x2), x2.shape[0], x2.shape[1], _ptr(out))
    return out


def sample(sampler, logits: torch.Tensor) -> torch.Tensor:
    """Sampler::sample (sampler.rs:22-37) on the device over one row of f32
    logits; returns the token as a one-element int32 device tensor and moves
    the sampler's stream past the draw the kernel took."""
    x = logits.contiguous().reshape(-1)
    if x.dtype != torch.float32:
        raise TypeError("logits must be float32")
    out = torch.empty(1, dtype=torch.int32, device=logits.device)
    call("prana_sample_logits", context(logits.device.index), _ptr(x), x.numel(), sampler.handle, _ptr(out))
    return out
