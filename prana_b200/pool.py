"""BufferPool (crates/prana-tensor/src/pool.rs:13-103) over the library's
device arena: one reservation, power-of-two buckets of at least 1 KiB,
released buffers recycled per bucket, the reference's active / pooled / peak
counters.  Attached to a device's context, it also backs every weight, model,
KV cache and scratch buffer the library allocates there."""
from __future__ import annotations

import ctypes as C

from . import _ffi
from ._ffi import call


class BufferPool:
    def __init__(self, capacity: int, device: int | None = None):
        """capacity bytes reserved on `device` (None: host memory, for bookkeeping)."""
        self._h = C.c_void_p()
        ctx = None
        if device is not None:
            from .kernels import context

            ctx = context(device)
        self.device = device
        call("prana_pool_create", ctx, capacity, C.byref(self._h))

    def acquire(self, byte_size: int) -> tuple[int, int]:
        """A zeroed buffer of at least byte_size bytes: (address, bucket bytes);
        (0, 0) for a zero-byte request."""
        p, got = C.c_void_p(), C.c_size_t()
        call("prana_pool_acquire", self._h, byte_size, C.byref(p), C.byref(got))
        return p.value or 0, got.value

    def release(self, address: int) -> None:
        call("prana_pool_release", self._h, C.c_void_p(address))

    def clear(self) -> None:
        call("prana_pool_clear", self._h)

    def _stats(self):
        v = [C.c_size_t() for _ in range(4)]
        call("prana_pool_stats", self._h, *[C.byref(x) for x in v])
        return [x.value for x in v]

    def active_bytes(self) -> int:
        return self._stats()[0]

    def pooled_bytes(self) -> int:
        return self._stats()[1]

    def peak_bytes(self) -> int:
        return self._stats()[2]

    def carved_bytes(self) -> int:
        return self._stats()[3]

    def attach(self) -> None:
        """Make this device's context allocate from the pool."""
        from .kernels import context

        call("prana_ctx_use_pool", context(self.device), self._h)

    def detach(self) -> None:
        from .kernels import context

        call("prana_ctx_use_pool", context(self.device), None)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _ffi.lib().prana_pool_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
