"""Seeded random-init models and quantized matrices (host-only, libprana_synth.so).

There is no network for checkpoints, so every model the benchmarks and parity
tests use is generated here from a seed in the shape of one of the reference
configurations.  `write_gguf` writes a GGUF v3 file the reference loader reads
(tensor names and metadata keys of gguf.rs:338-460).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import asdict, dataclass, replace
from pathlib import Path

import numpy as np

from ._ffi import TYPE_F32, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libprana_synth.so"


class _SynthModel(C.Structure):
    _fields_ = [
        ("arch", C.c_char * 16),
        ("dim", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("ctx", C.c_int),
        ("rope_theta", C.c_float), ("eps", C.c_float),
        ("has_bias", C.c_int), ("tied", C.c_int),
        ("type_embd", C.c_int), ("type_q", C.c_int), ("type_k", C.c_int), ("type_v", C.c_int),
        ("type_o", C.c_int), ("type_gate", C.c_int), ("type_up", C.c_int), ("type_down", C.c_int),
        ("type_output", C.c_int),
        ("seed", C.c_uint64),
        ("std", C.c_float), ("out_proj_mult", C.c_float), ("embd_std_mult", C.c_float), ("head_std_mult", C.c_float),
        ("code_rank", C.c_int), ("code_seed", C.c_uint64), ("code_noise", C.c_float),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; run `python -m prana_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        L.synth_write_gguf.argtypes = [C.POINTER(_SynthModel), C.c_char_p, C.c_int]
        L.synth_write_gguf.restype = C.c_int
        L.synth_tensor.argtypes = [C.c_int, C.c_size_t, C.c_size_t, C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                   C.c_int, C.c_void_p]
        L.synth_tensor.restype = C.c_int
        L.synth_encode_row.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
        L.synth_encode_row.restype = C.c_int
        L.synth_row_bytes.argtypes = [C.c_int, C.c_size_t]
        L.synth_row_bytes.restype = C.c_size_t
        L.synth_normal_row.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_size_t, C.c_float, C.c_void_p]
        L.synth_normal_row.restype = None
        _lib = L
    return _lib


@dataclass(frozen=True)
class ModelSpec:
    arch: str
    dim: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    ctx: int
    rope_theta: float
    eps: float = 0.0  # <= 0: metadata key omitted (loader default 1e-5)
    has_bias: bool = False
    tied: bool = False
    type_embd: int = TYPE_Q8_0
    type_q: int = TYPE_Q8_0
    type_k: int = TYPE_Q8_0
    type_v: int = TYPE_Q8_0
    type_o: int = TYPE_Q8_0
    type_gate: int = TYPE_Q8_0
    type_up: int = TYPE_Q8_0
    type_down: int = TYPE_Q8_0
    type_output: int = TYPE_Q8_0
    seed: int = 1234
    std: float = 0.02
    out_proj_mult: float = 1.0
    embd_std_mult: float = 1.0
    head_std_mult: float = 1.0
    # shared-code construction (synth.h): embedding and head rows from a token code
    # shared by every model with the same code_seed; code_noise sets how often two
    # such models pick different greedy tokens
    code_rank: int = 0
    code_seed: int = 0
    code_noise: float = 0.0

    def with_types(self, t: int) -> "ModelSpec":
        return replace(self, type_embd=t, type_q=t, type_k=t, type_v=t, type_o=t, type_gate=t, type_up=t,
                       type_down=t, type_output=t)

    def weight_bytes_per_token(self) -> int:
        """GGUF bytes of every matrix a decode step streams (embedding row excluded)."""
        rb = lambda t, cols: int(lib().synth_row_bytes(t, cols))
        q_dim, kv_dim = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        per_layer = (q_dim * rb(self.type_q, self.dim) + kv_dim * rb(self.type_k, self.dim)
                     + kv_dim * rb(self.type_v, self.dim) + self.dim * rb(self.type_o, q_dim)
                     + self.hidden * rb(self.type_gate, self.dim) + self.hidden * rb(self.type_up, self.dim)
                     + self.dim * rb(self.type_down, self.hidden))
        head = self.vocab * rb(self.type_embd if self.tied else self.type_output, self.dim)
        return per_layer * self.n_layers + head


# ---- the BASELINE configurations ----------------------------------------------------------

# C1: stories15M shape, Q8_0 everywhere (llama arch: interleaved RoPE)
STORIES15M_Q8 = ModelSpec("llama", 288, 768, 6, 6, 6, 48, 32000, 256, 10000.0, 1e-5)

# C3: Qwen2-0.5B shape, Q4_K_M-style mixture.  K-quants need cols % 256 == 0
# (kquant.rs:168), so only ffn_down (cols 4864) can be Q6_K; the cols-896 slots
# fall back to 32-block types (Q4_K -> Q4_0, Q6_K -> Q8_0).
QWEN2_0P5B_MIX = ModelSpec("qwen2", 896, 4864, 24, 14, 2, 64, 151936, 4096, 1e6, 1e-6, has_bias=True,
                           type_embd=TYPE_Q4_0, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q8_0,
                           type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q6_K,
                           type_output=TYPE_Q8_0)

# C4: Llama-3-8B shape (Q4_0 and Q8_0 variants)
LLAMA3_8B_Q4_0 = ModelSpec("llama", 4096, 14336, 32, 32, 8, 128, 128256, 8192, 5e5, 1e-5).with_types(TYPE_Q4_0)
LLAMA3_8B_Q8_0 = LLAMA3_8B_Q4_0.with_types(TYPE_Q8_0)
# Profiling case: the 8B layer shapes with 4 layers (~0.8 GB of weights, still
# far larger than L2), for captures that must hold little device memory.
LLAMA3_8B_Q4_0_L4 = replace(LLAMA3_8B_Q4_0, n_layers=4)
# Parity cases at the benchmarked width: every 8B tensor shape (dim 4096,
# 32/8 heads, FFN 14336, vocab 128256) with 2 layers, so the CPU oracle keeps
# up.
LLAMA3_8B_Q4_0_L2 = replace(LLAMA3_8B_Q4_0, n_layers=2)
LLAMA3_8B_Q8_0_L2 = replace(LLAMA3_8B_Q8_0, n_layers=2)

# C5: Qwen2 shapes for speculative decode (Q8_0)
QWEN2_0P5B_Q8 = replace(QWEN2_0P5B_MIX.with_types(TYPE_Q8_0), ctx=4096)
QWEN2_1P5B_Q8 = ModelSpec("qwen2", 1536, 8960, 28, 12, 2, 128, 151936, 4096, 1e6, 1e-6, has_bias=True).with_types(TYPE_Q8_0)

# C5 speculative pair at context 1024: both models near-bigram (block outputs
# scaled by out_proj_mult) over a shared token code, per-model noise tuned so
# the greedy draft's tokens are accepted about 60% of the time
C5_CODE = dict(code_rank=64, code_seed=2024, out_proj_mult=0.05)
C5_NOISE = 1.75  # measured on B200: 1.7 -> 67 %, 1.8 -> 54 % of drafted tokens accepted
QWEN2_0P5B_Q8_SPEC = replace(QWEN2_0P5B_Q8, ctx=1024, seed=1201, code_noise=C5_NOISE, **C5_CODE)
QWEN2_1P5B_Q8_SPEC = replace(QWEN2_1P5B_Q8, ctx=1024, seed=1501, code_noise=C5_NOISE, **C5_CODE)

PRESETS = {
    "stories15m_q8_0": STORIES15M_Q8,
    "qwen2_0p5b_mix": QWEN2_0P5B_MIX,
    "llama3_8b_q4_0": LLAMA3_8B_Q4_0,
    "llama3_8b_q8_0": LLAMA3_8B_Q8_0,
    "llama3_8b_q4_0_l4": LLAMA3_8B_Q4_0_L4,
    "llama3_8b_q4_0_l2": LLAMA3_8B_Q4_0_L2,
    "llama3_8b_q8_0_l2": LLAMA3_8B_Q8_0_L2,
    "qwen2_0p5b_q8_0": QWEN2_0P5B_Q8,
    "qwen2_1p5b_q8_0": QWEN2_1P5B_Q8,
    "qwen2_0p5b_q8_0_spec": QWEN2_0P5B_Q8_SPEC,
    "qwen2_1p5b_q8_0_spec": QWEN2_1P5B_Q8_SPEC,
}


def write_gguf(spec: ModelSpec, path: str | os.PathLike, threads: int | None = None) -> Path:
    d = asdict(spec)
    s = _SynthModel()
    s.arch = spec.arch.encode()
    for k, v in d.items():
        if k == "arch":
            continue
        setattr(s, k, int(v) if isinstance(v, bool) else v)
    threads = threads or min(os.cpu_count() or 1, 64)
    rc = lib().synth_write_gguf(C.byref(s), str(path).encode(), threads)
    if rc != 0:
        raise RuntimeError(f"synth_write_gguf failed with {rc}")
    return Path(path)


def normal_rows(seed: int, tensor: int, rows: int, cols: int, std: float = 0.02) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float32)
    for r in range(rows):
        lib().synth_normal_row(seed, tensor, r, cols, std, out[r].ctypes.data_as(C.c_void_p))
    return out


def encode(ggml_type: int, x: np.ndarray) -> np.ndarray:
    """Encode f32 rows [rows, cols] into GGUF block bytes [rows, row_bytes]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    rb = int(lib().synth_row_bytes(ggml_type, cols))
    if rb == 0:
        raise ValueError(f"type {ggml_type} cannot hold {cols} columns")
    out = np.empty((rows, rb), dtype=np.uint8)
    for r in range(rows):
        if lib().synth_encode_row(ggml_type, x[r].ctypes.data_as(C.c_void_p), cols, out[r].ctypes.data_as(C.c_void_p)):
            raise RuntimeError("encode failed")
    return out


def matrix(ggml_type: int, rows: int, cols: int, seed: int, tensor: int = 1, std: float = 0.02,
           threads: int | None = None) -> np.ndarray:
    """A seeded N(0, std) matrix encoded as GGUF blocks: [rows, row_bytes] uint8."""
    rb = int(lib().synth_row_bytes(ggml_type, cols))
    if rb == 0:
        raise ValueError(f"type {ggml_type} cannot hold {cols} columns")
    out = np.empty((rows, rb), dtype=np.uint8)
    rc = lib().synth_tensor(ggml_type, rows, cols, seed, tensor, std, 0.0, threads or min(os.cpu_count() or 1, 64),
                            out.ctypes.data_as(C.c_void_p))
    if rc:
        raise RuntimeError("synth_tensor failed")
    return out
