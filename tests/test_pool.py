"""The buffer pool's bookkeeping (CPU only, host-memory arena): the
reference's own pool tests (crates/prana-tensor/src/pool.rs:104-121) restated,
plus the arena behaviour -- zeroed buffers, exhaustion as an error, clear()
returning cached buffers to a coalescing arena."""
import ctypes as C

import pytest

from prana_b200._ffi import PranaError
from prana_b200.pool import BufferPool


def test_recycles_same_bucket():
    pool = BufferPool(1 << 20)
    a, size = pool.acquire(2000)
    assert size == 2048
    assert pool.active_bytes() == 2048
    pool.release(a)
    assert pool.active_bytes() == 0
    assert pool.pooled_bytes() == 2048
    # a second acquire of the same bucket reuses the buffer, not the arena
    b, size = pool.acquire(1500)
    assert size == 2048 and b == a
    assert pool.pooled_bytes() == 0
    assert pool.peak_bytes() == 2048


def test_zero_is_free():
    pool = BufferPool(1 << 20)
    assert pool.acquire(0) == (0, 0)


def test_buckets_and_large_requests():
    pool = BufferPool(300 << 20)
    assert pool.acquire(1)[1] == 1024
    assert pool.acquire(1025)[1] == 2048
    assert pool.acquire(5000)[1] == 8192
    big = (64 << 20) + 1000  # above the bucket range: its own 256-byte-aligned size
    assert pool.acquire(big)[1] == (big + 255) // 256 * 256


def test_buffers_are_zeroed_on_acquire():
    pool = BufferPool(1 << 20)
    a, n = pool.acquire(4096)
    C.memset(a, 0x5A, n)
    pool.release(a)
    b, n = pool.acquire(4096)
    assert b == a and C.string_at(b, n) == bytes(n)


def test_exhaustion_is_an_error():
    pool = BufferPool(16 << 10)
    pool.acquire(8 << 10)
    pool.acquire(8 << 10)
    with pytest.raises(PranaError, match="PRANA_E_OOM"):
        pool.acquire(1024)


def test_clear_returns_buffers_to_a_coalescing_arena():
    cap = 64 << 10
    pool = BufferPool(cap)
    bufs = [pool.acquire(16 << 10)[0] for _ in range(4)]
    assert pool.carved_bytes() == cap
    for b in bufs:
        pool.release(b)
    with pytest.raises(PranaError):  # cached in the 16 KiB bucket: no room for a 32 KiB buffer
        pool.acquire(32 << 10)
    pool.clear()
    assert pool.pooled_bytes() == 0 and pool.carved_bytes() == 0
    whole, n = pool.acquire(cap)  # the four ranges merged back into one
    assert n == cap and whole == bufs[0]


def test_foreign_and_double_release_are_errors():
    pool = BufferPool(1 << 20)
    a, _ = pool.acquire(1024)
    pool.release(a)
    with pytest.raises(PranaError, match="not checked out"):
        pool.release(a)
    with pytest.raises(PranaError, match="does not belong"):
        pool.release(a + (2 << 20))
