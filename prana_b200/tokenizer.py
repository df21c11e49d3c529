"""Prompt encoding and token decoding over the library's host-side tokenizers:
SentencePiece-style greedy BPE (tokenizer.rs) and GPT-2 byte-level BPE
(bpe.rs), built from a GGUF file's metadata (gguf.rs:462-537) or from piece
lists.  Nothing here touches a GPU."""
from __future__ import annotations

import ctypes as C

from ._ffi import call

BOS, EOS = 1, 2  # tokenizer.rs:15-16 defaults


def _strings(items):
    bs = [s.encode() if isinstance(s, str) else bytes(s) for s in items]
    bufs = [C.create_string_buffer(b, len(b) + 1) for b in bs]
    ptrs = (C.c_char_p * len(bs))(*[C.cast(b, C.c_char_p) for b in bufs])
    lens = (C.c_size_t * len(bs))(*[len(b) for b in bs])
    return bufs, ptrs, lens


class Tokenizer:
    def __init__(self, handle: C.c_void_p):
        self._h = handle

    @classmethod
    def load_gguf(cls, path: str) -> "Tokenizer":
        """load_tokenizer (gguf.rs:462-537)."""
        h = C.c_void_p()
        call("prana_tokenizer_load_gguf", str(path).encode(), C.byref(h))
        return cls(h)

    @classmethod
    def spm(cls, pieces, scores, bos: int = BOS, eos: int = EOS, add_bos: bool = True) -> "Tokenizer":
        """Tokenizer::from_parts + with_special (tokenizer.rs:51-67); pieces are bytes or str."""
        assert len(pieces) == len(scores)
        keep, ptrs, lens = _strings(pieces)
        sc = (C.c_float * len(scores))(*scores)
        h = C.c_void_p()
        call("prana_tokenizer_spm", len(pieces), ptrs, lens, sc, bos, eos, int(add_bos), C.byref(h))
        del keep
        return cls(h)

    @classmethod
    def bpe(cls, vocab, merges, bos=None, eos=None, add_bos: bool = False, specials=()) -> "Tokenizer":
        """BpeTokenizer::new + with_specials (bpe.rs:57-84); specials are vocab ids."""
        kv, vp, vl = _strings(vocab)
        km, mp, ml = _strings(merges)
        sp = (C.c_uint32 * max(len(specials), 1))(*specials)
        h = C.c_void_p()
        call("prana_tokenizer_bpe", len(vocab), vp, vl, len(merges), mp, ml, len(specials), sp,
             -1 if bos is None else bos, -1 if eos is None else eos, int(add_bos), C.byref(h))
        del kv, km
        return cls(h)

    @property
    def vocab_size(self) -> int:
        n = C.c_size_t()
        call("prana_tokenizer_vocab_size", self._h, C.byref(n))
        return n.value

    def encode(self, text, bos: bool | None = None, eos: bool = False) -> list[int]:
        """encode_prompt when bos is None; SentencePiece's encode(text, bos, eos) otherwise."""
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = C.c_size_t()
        cap = 2 * len(b) + 8
        out = (C.c_uint32 * cap)()
        call("prana_tokenize", self._h, b, len(b), -1 if bos is None else int(bos), int(eos), out, cap, C.byref(n))
        return list(out[: n.value])

    def decode(self, prev: int, token: int) -> bytes:
        """The bytes of one token given the previous one (Tokenize::decode)."""
        n = C.c_size_t()
        cap = 256
        out = C.create_string_buffer(cap)
        try:
            call("prana_detokenize", self._h, prev, token, out, cap, C.byref(n))
        except RuntimeError:
            if n.value <= cap:
                raise
            out = C.create_string_buffer(n.value)
            call("prana_detokenize", self._h, prev, token, out, n.value, C.byref(n))
        return out.raw[: n.value]

    def is_stop(self, token: int) -> bool:
        r = C.c_int()
        call("prana_tokenizer_is_stop", self._h, token, C.byref(r))
        return bool(r.value)

    def close(self):
        if self._h:
            call("prana_tokenizer_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
