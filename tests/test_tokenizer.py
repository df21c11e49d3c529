"""The host-side tokenizers against the reference's own tokenizer tests (CPU only).

SentencePiece-style: crates/prana-model/src/tokenizer.rs:233-269 (greedy merges
with the dummy prefix, byte fallback, decode after BOS and of <0xNN> pieces).
Byte-level BPE: crates/prana-model/src/bpe.rs:205-274 (rank order, byte round
trip, stop ids, the leading-space pre-split, verbatim special tokens).
GGUF metadata: gguf.rs:462-537 (model selection, U+2581 pieces, defaults),
through small GGUF files written here.
"""
import struct

import numpy as np
import pytest

from prana_b200._ffi import PranaError
from prana_b200.tokenizer import BOS, Tokenizer


def spm(entries, **kw):
    return Tokenizer.spm([p for _, p in entries], [s for s, _ in entries], **kw)


def tiny_spm():
    return spm([(0.0, b"<unk>"), (0.0, b"<s>"), (0.0, b"</s>"), (-1.0, b" "), (-2.0, b"h"), (-2.0, b"i"),
                (-1.5, b"hi"), (-1.2, b" hi")])


def test_spm_greedy_merges_and_dummy_prefix():
    # " " + "h" + "i" -> "hi" (-1.5) first, then " " + "hi" -> " hi" (-1.2)
    assert tiny_spm().encode("hi", bos=True) == [BOS, 7]


def test_spm_byte_fallback():
    # dummy prefix " " (id 3), then 'z' = 0x7A through the byte fallback (+3)
    assert tiny_spm().encode("z", bos=False) == [3, ord("z") + 3]


def test_spm_decode_after_bos_and_byte_pieces():
    t = spm([(0.0, b"<unk>"), (0.0, b"<s>"), (0.0, b"</s>"), (-1.0, b" word"), (0.0, b"<0x0A>")])
    assert t.decode(BOS, 3) == b"word"
    assert t.decode(9, 3) == b" word"
    assert t.decode(3, 4) == b"\n"
    assert t.is_stop(1) and t.is_stop(2) and not t.is_stop(3)


def test_spm_encode_prompt_adds_bos_and_eos_on_request():
    t = tiny_spm()
    assert t.encode("hi") == [BOS, 7]  # add_bos defaults on
    assert t.encode("hi", bos=False, eos=True) == [7, 2]
    assert t.encode("", bos=False) == []  # no dummy prefix for empty text


def byte_fallback_spm():
    pieces = [b"<unk>", b"<s>", b"</s>"] + [b"<0x%02X>" % b for b in range(256)] + [b" ", b"a", b"b", b" ab"]
    scores = [0.0] * len(pieces)
    scores[-1] = 1.0
    return Tokenizer.spm(pieces, scores), pieces


def test_spm_byte_round_trip():
    t, _ = byte_fallback_spm()
    rng = np.random.default_rng(5)
    for _ in range(20):
        text = "".join(rng.choice(list("ab xé€😀\n"), size=int(rng.integers(1, 12))))
        ids = t.encode(text, bos=True)
        out, prev = b"", ids[0]
        for i in ids[1:]:
            out += t.decode(prev, i)
            prev = i
        assert out == text.encode(), (text, ids)


# ---- byte-level BPE (bpe.rs) ---------------------------------------------------------------


def bytes_to_unicode():
    table, n = [], 0
    for b in range(256):
        if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
            table.append(chr(b))
        else:
            table.append(chr(256 + n))
            n += 1
    return table


SP = bytes_to_unicode()[ord(" ")]  # 'Ġ'


def tiny_bpe(specials=()):
    vocab = ["h", "i", SP, "hi", SP + "hi", "<|endoftext|>"]
    return Tokenizer.bpe(vocab, ["h i", f"{SP} hi"], bos=None, eos=5, add_bos=False, specials=specials)


def test_bpe_merges_in_rank_order():
    t = tiny_bpe()
    assert t.encode("hi") == [3]
    assert t.encode(" hi") == [4]


def test_bpe_decode_round_trips_bytes():
    t = tiny_bpe()
    assert b"".join(t.decode(0, i) for i in t.encode(" hi")) == b" hi"


def test_bpe_eos_is_stop():
    t = tiny_bpe()
    assert t.is_stop(5) and not t.is_stop(3)


def test_bpe_pre_split_keeps_leading_spaces_on_words():
    # merges that build every piece of "hello world 42!" whole; the pre-split
    # must give exactly ["hello", " world", " 42", "!"]
    enc = bytes_to_unicode()
    vocab = list(enc)
    merges = []
    for word in ["hello", " world", " 42"]:
        syms = "".join(enc[b] for b in word.encode())
        for k in range(2, len(syms) + 1):
            merges.append(f"{syms[:k - 1]} {syms[k - 1]}")
            vocab.append(syms[:k])
    t = Tokenizer.bpe(vocab, merges)
    ids = t.encode("hello world 42!")
    want = ["hello", SP + "world", SP + "42", "!"]
    assert ids == [vocab.index(w) for w in want]


def test_bpe_merges_never_cross_the_pre_split():
    enc = bytes_to_unicode()
    vocab = list(enc) + ["o" + SP]
    t = Tokenizer.bpe(vocab, [f"o {SP}"])
    assert len(vocab) - 1 not in t.encode("lo w")  # "lo" | " w": the o-space merge cannot fire


def test_bpe_specials_encode_verbatim():
    t = tiny_bpe(specials=[5])
    assert t.encode("hi<|endoftext|> hi") == [3, 5, 4]
    assert t.encode("<|endoftext|>") == [5]
    assert tiny_bpe().encode("hi<|endoftext|> hi") != [3, 5, 4]


def test_bpe_byte_round_trip():
    t = Tokenizer.bpe(bytes_to_unicode(), [])
    for text in ["plain ascii", "naïve café", "日本語 テキスト", "emoji 😀 ok", "tabs\tand\nnewlines"]:
        assert b"".join(t.decode(0, i) for i in t.encode(text)) == text.encode()


def test_invalid_utf8_is_replaced_like_from_utf8_lossy():
    t = Tokenizer.bpe(bytes_to_unicode(), [])
    # 0xFF is never valid; E2 82 (a truncated 3-byte sequence) is one maximal subpart
    got = b"".join(t.decode(0, i) for i in t.encode(b"a\xffb\xe2\x82c"))
    assert got == "a�b�c".encode()


# ---- GGUF metadata (gguf.rs:462-537) -------------------------------------------------------


def gguf_bytes(kvs):
    """A GGUF v3 file holding only metadata (no tensors)."""
    def s(x):
        b = x.encode() if isinstance(x, str) else x
        return struct.pack("<Q", len(b)) + b

    out = b"GGUF" + struct.pack("<IQQ", 3, 0, len(kvs))
    for key, ty, val in kvs:
        out += s(key) + struct.pack("<I", ty)
        if ty == 8:
            out += s(val)
        elif ty == 4:
            out += struct.pack("<I", val)
        elif ty == 5:
            out += struct.pack("<i", val)
        elif ty == 7:
            out += struct.pack("<B", int(val))
        elif ty == 9:
            et, items = val
            out += struct.pack("<IQ", et, len(items))
            for it in items:
                out += s(it) if et == 8 else struct.pack({6: "<f", 4: "<I", 5: "<i"}[et], it)
    return out


def test_gguf_llama_tokenizer(tmp_path):
    toks = ["<unk>", "<s>", "</s>", "▁", "h", "i", "hi", "▁hi"]
    path = tmp_path / "spm.gguf"
    path.write_bytes(gguf_bytes([
        ("tokenizer.ggml.model", 8, "llama"),
        ("tokenizer.ggml.tokens", 9, (8, toks)),
        ("tokenizer.ggml.scores", 9, (6, [0, 0, 0, -1, -2, -2, -1.5, -1.2])),
        ("tokenizer.ggml.bos_token_id", 4, 1),
        ("tokenizer.ggml.eos_token_id", 4, 2),
    ]))
    t = Tokenizer.load_gguf(path)
    assert t.vocab_size == len(toks)
    assert t.encode("hi") == [1, 7]  # U+2581 pieces read as spaces; BOS added by default
    assert t.decode(1, 7) == b"hi"


def test_gguf_gpt2_tokenizer(tmp_path):
    toks = ["h", "i", SP, "hi", SP + "hi", "<|im_end|>"]
    path = tmp_path / "bpe.gguf"
    path.write_bytes(gguf_bytes([
        ("tokenizer.ggml.model", 8, "gpt2"),
        ("tokenizer.ggml.tokens", 9, (8, toks)),
        ("tokenizer.ggml.merges", 9, (8, ["h i", f"{SP} hi"])),
        ("tokenizer.ggml.token_type", 9, (5, [1, 1, 1, 1, 1, 3])),
        ("tokenizer.ggml.eos_token_id", 4, 5),
    ]))
    t = Tokenizer.load_gguf(path)
    assert t.encode("hi<|im_end|> hi") == [3, 5, 4]  # no BOS: gpt2 defaults to none
    assert t.is_stop(5)


def test_gguf_rejects_unknown_model_and_missing_merges(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(gguf_bytes([("tokenizer.ggml.model", 8, "wordpiece"), ("tokenizer.ggml.tokens", 9, (8, ["a"]))]))
    with pytest.raises(PranaError, match="unsupported tokenizer"):
        Tokenizer.load_gguf(bad)
    nomerge = tmp_path / "nomerge.gguf"
    nomerge.write_bytes(gguf_bytes([("tokenizer.ggml.model", 8, "gpt2"), ("tokenizer.ggml.tokens", 9, (8, ["a"]))]))
    with pytest.raises(PranaError, match="merges"):
        Tokenizer.load_gguf(nomerge)
