"""The C ABI without a GPU (CPU only): the library loads, exports every entry
point include/prana_cuda.h declares, and reports errors through status codes
and prana_last_error() instead of crashing."""
import ctypes as C
import re
from pathlib import Path

import pytest

from prana_b200 import _ffi
from prana_b200 import build as pbuild

HEADER = Path(__file__).resolve().parent.parent / "include" / "prana_cuda.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return sorted(set(re.findall(r"\b(prana_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not _ffi.LIB_PATH.exists():
        pbuild.build_all()
    return C.CDLL(str(_ffi.LIB_PATH))


def test_header_declares_the_surface():
    names = declared_functions()
    for required in ["prana_ctx_create", "prana_weight_upload", "prana_quantize_acts", "prana_matmul_kquant_f32",
                     "prana_attention_decode", "prana_model_load_gguf", "prana_forward", "prana_generate"]:
        assert required in names, required
    assert len(names) >= 40


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared in {HEADER.name} but not exported: {missing}"


def test_errors_are_codes_not_crashes(lib):
    lib.prana_last_error.restype = C.c_char_p
    lib.prana_ctx_create.argtypes = [C.c_int, C.POINTER(C.c_void_p)]
    ctx = C.c_void_p()
    rc = lib.prana_ctx_create(-1, C.byref(ctx))  # no such device, with or without a GPU
    assert rc < 0
    assert lib.prana_last_error()
    lib.prana_ctx_destroy.argtypes = [C.c_void_p]
    assert lib.prana_ctx_destroy(None) == 0  # destroying nothing is a no-op
