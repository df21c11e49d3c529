"""Token sampling (sampler.rs): greedy argmax, or temperature sampling with
the reference's seeded xorshift64* stream.  Sampler.sample runs on host
logits; the same sampler drives the device forms (prana_b200.kernels.sample,
prana_b200.model.generate_sampled and DecodeLoop.begin(..., sampler=))."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._ffi import call


class Sampler:
    def __init__(self, temperature: float = 0.0, seed: int = 0):
        """Sampler::new (sampler.rs:13-20): greedy when temperature <= 0."""
        self.greedy = temperature <= 0.0  # NaN samples, as in the reference
        self._h = C.c_void_p()
        call("prana_sampler_create", float(temperature), int(seed) & (2**64 - 1), C.byref(self._h))

    def sample(self, logits) -> int:
        """Sampler::sample (sampler.rs:22-37) over one row of logits."""
        x = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)
        t = C.c_uint32()
        call("prana_sample", self._h, x.ctypes.data_as(C.c_void_p), x.size, C.byref(t))
        return t.value

    @property
    def handle(self):
        return self._h

    def next_f32(self) -> float:
        """XorShift::next_f32: the stream's next uniform draw in [0, 1)."""
        v = C.c_float()
        call("prana_sampler_next_f32", self._h, C.byref(v))
        return v.value

    def close(self):
        if self._h:
            call("prana_sampler_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
