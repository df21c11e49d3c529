"""generate_text's host loop (infer.rs:696-771) with a stand-in model (CPU
only): prompt prefill and teacher forcing, which positions read logits, the
stop id, the context limit, and the greedy / sampled successor."""
from dataclasses import dataclass

import numpy as np
import pytest

from prana_b200 import generate as gen
from prana_b200 import model as pm
from prana_b200.sampler import Sampler
from prana_b200.tokenizer import Tokenizer


def bytes_to_unicode():
    table, n = [], 0
    for b in range(256):
        if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
            table.append(chr(b))
        else:
            table.append(chr(256 + n))
            n += 1
    return table


EOS = 256


def tokenizer():
    # byte-level vocabulary: id = byte value, plus an end-of-sequence token
    return Tokenizer.bpe(bytes_to_unicode() + ["<eos>"], [], eos=EOS)


@dataclass
class Cfg:
    seq_len: int
    vocab_size: int = 257


class FakeModel:
    def __init__(self, seq_len):
        self.config = Cfg(seq_len)
        self.calls = []  # (token, pos, want_logits)


@pytest.fixture
def fake(monkeypatch):
    """prefill / forward of a model whose successor of byte t is t + 1 up to 'e' (then EOS)."""
    class Cache:
        def __init__(self, model, n):
            self.n = n

        def close(self):
            pass

    def successor(t):
        return t + 1 if t + 1 < ord("e") else EOS

    def forward(model, cache, token, pos, want_logits=True):
        assert pos < cache.n
        model.calls.append((token, pos, want_logits))
        nxt = successor(token)
        logits = np.zeros(model.config.vocab_size, np.float32)
        logits[nxt] = 50.0
        return (logits if want_logits else None), nxt

    def forward_sampled(model, cache, token, pos, sampler):
        # the device sampler over the step's logits, stood in by the host sampler
        assert pos < cache.n
        model.calls.append((token, pos, "sampled"))
        logits = np.zeros(model.config.vocab_size, np.float32)
        logits[successor(token)] = 50.0
        return sampler.sample(logits)

    prefilled = []
    monkeypatch.setattr(pm, "forward_sampled", forward_sampled)
    monkeypatch.setattr(pm, "KvCache", Cache)
    monkeypatch.setattr(pm, "prefill", lambda model, cache, toks: prefilled.append(list(toks)))
    monkeypatch.setattr(pm, "forward", forward)
    return prefilled


def test_greedy_continues_until_the_stop_id(fake):
    m, streamed = FakeModel(64), []
    out, st = gen.generate_text(m, tokenizer(), "ab", 10, on_piece=lambda b, p: streamed.append((b, p)))
    assert out == b"cd" and (st.prompt_tokens, st.generated_tokens) == (2, 2)
    assert fake == [[ord("a")]]  # all but the last prompt token, in one batch
    assert streamed == [(b"b", True), (b"c", False), (b"d", False)]
    # greedy reads the device argmax: no logits copied back
    assert [c[2] for c in m.calls] == [False, False, False]
    assert [c[1] for c in m.calls] == [1, 2, 3]


def test_context_limit_stops_before_the_next_position(fake):
    m = FakeModel(3)
    out, st = gen.generate_text(m, tokenizer(), "ab", 10)
    assert out == b"c" and st.generated_tokens == 1
    assert [c[1] for c in m.calls] == [1, 2]


def test_sampled_positions_sample_on_the_device(fake):
    m = FakeModel(64)
    out, _ = gen.generate_text(m, tokenizer(), "abc", 10, sampler=Sampler(0.5, 9))
    assert out == b"d"  # the logits put (almost) all mass on the successor
    # positions whose successor is sampled draw it beside their logits (no logits
    # copied back); the last position does not exist
    assert [(c[1], c[2]) for c in m.calls] == [(2, "sampled"), (3, "sampled")]


def test_empty_prompt_is_rejected(fake):
    with pytest.raises(ValueError):
        gen.generate_text(FakeModel(8), tokenizer(), "", 4)
