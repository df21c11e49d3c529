"""The device arena backing a context (GPU): with a BufferPool attached, a
model's weights, KV caches, activation buffers and kernel scratch are carved
from the pool's one reservation (no allocator call after it), and the model
computes exactly what it computes without the pool."""
import numpy as np
import pytest
import torch

from prana_b200 import kernels as K
from prana_b200 import model as pm
from prana_b200 import synth
from prana_b200._ffi import TYPE_Q4_0, PranaError
from prana_b200.pool import BufferPool

pytestmark = pytest.mark.gpu

SPEC = synth.ModelSpec("llama", 256, 768, 2, 4, 2, 64, 777, 96, 5e5, 1e-5, seed=71).with_types(TYPE_Q4_0)


@pytest.fixture(scope="module")
def path(tmp_path_factory, gpu):
    p = tmp_path_factory.mktemp("pool") / "m.gguf"
    synth.write_gguf(SPEC, p)
    return p


def run(model):
    kv = pm.KvCache(model, 32)
    pm.prefill(model, kv, np.array([5, 9, 13, 2, 7, 1, 3, 4, 8, 6, 10, 11], np.uint32))  # the tensor-core batch path
    outs = [pm.forward(model, kv, t, 12 + i)[0] for i, t in enumerate([3, 17, 40])]
    kv.close()
    return outs


def test_model_from_the_arena_matches(path):
    ref_model = pm.Model.load(str(path), 0)
    ref = run(ref_model)
    ref_model.close()
    pool = BufferPool(256 << 20, device=0)
    pool.attach()
    try:
        m = pm.Model.load(str(path), 0)
        loaded = pool.active_bytes()
        assert loaded >= m.config.weight_bytes  # weights, norms, buffers all came from the arena
        got = run(m)
        for a, b in zip(got, ref):
            assert np.array_equal(a, b)
        m.close()
        assert pool.active_bytes() < loaded  # freed buffers went back to the pool's lists
        assert pool.peak_bytes() >= loaded
    finally:
        pool.detach()
        pool.close()


def test_kernel_scratch_from_the_arena(gpu):
    nh, nkv, hd, pos = 32, 8, 128, 2047
    q = torch.randn(nh * hd, device="cuda")
    kc = torch.randn(pos + 1, nkv * hd, device="cuda").half().view(torch.int16)
    vc = torch.randn(pos + 1, nkv * hd, device="cuda").half().view(torch.int16)
    ref = K.attention_decode(q, kc, vc, pos, nh, nkv, hd)
    K.synchronize()
    pool = BufferPool(64 << 20, device=0)
    pool.attach()
    try:
        # a fresh context scratch is carved from the pool the first time a larger one is needed
        w = K.QuantMatrix(TYPE_Q4_0, 512, 4096, synth.matrix(TYPE_Q4_0, 512, 4096, seed=3))
        a = torch.randn(40, 4096, device="cuda")
        out = K.matmul_kquant_f32(a, w, 40)
        got = K.attention_decode(q, kc, vc, pos, nh, nkv, hd)
        K.synchronize()
        assert torch.equal(got, ref) and torch.isfinite(out).all()
        assert pool.active_bytes() > 0
        del w
    finally:
        pool.detach()
        pool.close()


def test_device_buffers_are_zeroed(gpu):
    """acquire returns zeroed device memory even when the buffer is a recycled one."""
    from cuda.bindings import runtime as rt

    pool = BufferPool(1 << 20, device=0)
    try:
        a, n = pool.acquire(4096)
        assert rt.cudaMemset(a, 0x5A, n)[0] == rt.cudaError_t.cudaSuccess
        torch.cuda.synchronize()
        pool.release(a)
        b, _ = pool.acquire(4096)
        assert b == a
        torch.cuda.synchronize()
        host = np.full(n, 0xFF, np.uint8)
        err, = rt.cudaMemcpy(host.ctypes.data, b, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert err == rt.cudaError_t.cudaSuccess
        assert not host.any()
    finally:
        pool.close()


def test_too_small_an_arena_fails_cleanly(path):
    pool = BufferPool(1 << 20, device=0)
    pool.attach()
    try:
        with pytest.raises(PranaError, match="PRANA_E_OOM"):
            pm.Model.load(str(path), 0)
    finally:
        pool.detach()
        pool.close()
    m = pm.Model.load(str(path), 0)  # the context works as before
    assert run(m)[0].shape == (SPEC.vocab,)
    m.close()
