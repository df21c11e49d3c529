"""ctypes binding of include/prana_cuda.h (libprana_cuda.so, built in-tree).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libprana_cuda.so"

PRANA_OK = 0
ERRORS = {
    -1: "PRANA_E_INVALID",
    -2: "PRANA_E_CUDA",
    -3: "PRANA_E_OOM",
    -4: "PRANA_E_FORMAT",
    -5: "PRANA_E_UNSUPPORTED",
    -6: "PRANA_E_TIMEOUT",
    -7: "PRANA_E_COMM",
}

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 2, 8, 12, 14
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}


class PranaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class ModelConfig(C.Structure):
    _fields_ = [
        ("dim", C.c_int64), ("hidden_dim", C.c_int64), ("n_layers", C.c_int64), ("n_heads", C.c_int64),
        ("n_kv_heads", C.c_int64), ("vocab_size", C.c_int64), ("seq_len", C.c_int64), ("head_dim", C.c_int64),
        ("rope_theta", C.c_float), ("norm_eps", C.c_float),
        ("rope_neox", C.c_int32), ("has_bias", C.c_int32), ("shared_classifier", C.c_int32),
        ("weight_bytes", C.c_int64),
    ]


P = C.c_void_p
SZ = C.c_size_t
I = C.c_int

# name -> (argtypes); every function returns int status except where noted
SIGNATURES = {
    "prana_version": [],
    "prana_ctx_create": [I, C.POINTER(P)],
    "prana_ctx_destroy": [P],
    "prana_ctx_set_stream": [P, P],
    "prana_ctx_synchronize": [P],
    "prana_ctx_stream": [P, C.POINTER(P)],
    "prana_debug_wait_timeout": [P, I, C.c_uint],
    "prana_pool_create": [P, SZ, C.POINTER(P)],
    "prana_pool_destroy": [P],
    "prana_pool_acquire": [P, SZ, C.POINTER(P), C.POINTER(SZ)],
    "prana_pool_release": [P, P],
    "prana_pool_clear": [P],
    "prana_pool_stats": [P, C.POINTER(SZ), C.POINTER(SZ), C.POINTER(SZ), C.POINTER(SZ)],
    "prana_ctx_use_pool": [P, P],
    "prana_weight_upload": [P, I, SZ, SZ, P, C.POINTER(P)],
    "prana_weight_free": [P],
    "prana_quantize_q8": [SZ, SZ, P, P, P],
    "prana_weight_upload_q8": [P, SZ, SZ, P, C.POINTER(P)],
    "prana_weight_bytes": [P, C.POINTER(SZ)],
    "prana_quantize_acts": [P, P, SZ, SZ, P, P, P],
    "prana_matmul_q8_f32": [P, P, P, SZ, P],
    "prana_matmul_kquant_f32": [P, P, P, SZ, P],
    "prana_matmul_q8_prefill": [P, P, P, P, SZ, P, P],
    "prana_matmul_kquant_prefill": [P, P, P, P, SZ, P, P],
    "prana_matmul_f32": [P, P, P, SZ, P],
    "prana_qgemm": [P, P, P, P, SZ, P, P],
    "prana_qgemm_block_dots": [P, P, P, P, SZ, P, P],
    "prana_block_dots": [P, P, SZ, P, P, P],
    "prana_rmsnorm": [P, P, P, SZ, SZ, C.c_float, P],
    "prana_silu": [P, P, SZ],
    "prana_silu_mul": [P, P, P, SZ],
    "prana_softmax": [P, P, SZ, SZ, P],
    "prana_rope_interleaved": [P, P, SZ, SZ, SZ, SZ, C.c_float],
    "prana_rope_neox": [P, P, SZ, SZ, SZ, SZ, C.c_float],
    "prana_f16_kv_write": [P, P, SZ, SZ, P, SZ],
    "prana_attention_decode": [P, P, P, P, SZ, SZ, SZ, SZ, P],
    "prana_attention_decode_noalloc": [P, P, P, P, SZ, SZ, SZ, SZ, P],
    "prana_attention_verify": [P, P, P, P, SZ, SZ, SZ, SZ, SZ, P],
    "prana_attention": [P, P, P, P, SZ, SZ, SZ, SZ, P],
    "prana_argmax": [P, P, SZ, SZ, P],
    "prana_model_load_gguf": [P, C.c_char_p, C.POINTER(P)],
    "prana_model_load_gguf_ex": [P, C.c_char_p, I, C.POINTER(P)],
    "prana_model_load_gguf_tp": [P, C.c_char_p, I, I, P, C.POINTER(P)],
    "prana_tp_unique_id": [P],
    "prana_model_tp_get": [P, C.POINTER(I), C.POINTER(I), C.POINTER(I)],
    "prana_model_free": [P],
    "prana_model_config_get": [P, C.POINTER(ModelConfig)],
    "prana_kv_create": [P, SZ, C.POINTER(P)],
    "prana_kv_free": [P],
    "prana_kv_read": [P, SZ, I, SZ, P],
    "prana_kv_read_rows": [P, SZ, I, SZ, SZ, P],
    "prana_forward": [P, P, C.c_uint32, SZ, P, P],
    "prana_forward_trace": [P, P, C.c_uint32, SZ, P, P, P, SZ, C.POINTER(SZ)],
    "prana_kv_write": [P, SZ, I, SZ, P],
    "prana_forward_batch_trace": [P, P, P, SZ, SZ, I, P, P, P, SZ, C.POINTER(SZ)],
    "prana_prefill": [P, P, P, SZ],
    "prana_forward_batch": [P, P, P, SZ, SZ, P, P],
    "prana_forward_multi": [P, P, SZ, P, P, P, P],
    "prana_forward_multi_trace": [P, P, SZ, P, P, P, P, P, SZ, C.POINTER(SZ)],
    "prana_tokenizer_load_gguf": [C.c_char_p, C.POINTER(P)],
    "prana_tokenizer_spm": [SZ, P, P, P, C.c_uint32, C.c_uint32, I, C.POINTER(P)],
    "prana_tokenizer_bpe": [SZ, P, P, SZ, P, P, SZ, P, C.c_int64, C.c_int64, I, C.POINTER(P)],
    "prana_tokenizer_free": [P],
    "prana_tokenizer_vocab_size": [P, C.POINTER(SZ)],
    "prana_tokenize": [P, C.c_char_p, SZ, I, I, P, SZ, C.POINTER(SZ)],
    "prana_detokenize": [P, C.c_uint32, C.c_uint32, P, SZ, C.POINTER(SZ)],
    "prana_tokenizer_is_stop": [P, C.c_uint32, C.POINTER(I)],
    "prana_sampler_create": [C.c_float, C.c_uint64, C.POINTER(P)],
    "prana_sampler_free": [P],
    "prana_sample": [P, P, SZ, C.POINTER(C.c_uint32)],
    "prana_sampler_next_f32": [P, C.POINTER(C.c_float)],
    "prana_sample_logits": [P, P, SZ, P, P],
    "prana_generate_sampled": [P, P, SZ, SZ, C.c_int64, P, P, C.POINTER(SZ)],
    "prana_decode_begin_sampled": [P, P, C.c_uint32, SZ, P],
    "prana_forward_sampled": [P, P, C.c_uint32, SZ, P, C.POINTER(C.c_uint32)],
    "prana_generate": [P, P, SZ, SZ, C.c_int64, P, C.POINTER(SZ)],
    "prana_generate_speculative": [P, P, P, SZ, SZ, SZ, C.c_int64, P, C.POINTER(SZ), P],
    "prana_decode_begin": [P, P, C.c_uint32, SZ],
    "prana_decode_run": [P, P, SZ],
    "prana_decode_tokens": [P, P, P, SZ, C.POINTER(SZ)],
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it is missing: build it with prana_b200.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; run `python -m prana_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        L.prana_last_error.restype = C.c_char_p
        L.prana_last_error.argtypes = []
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = C.c_int
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != PRANA_OK:
        raise PranaError(rc, lib().prana_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
