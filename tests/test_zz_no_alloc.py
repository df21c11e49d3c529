"""prana_attention_decode_noalloc against prana_attention_decode (GPU).

The file name sorts last, so the suite also runs it after every other test has
used the library; it passes on its own as well.  Two calls in a row check that
the static ticket counters are left at zero by each call.
"""
import numpy as np
import pytest
import torch

from prana_b200 import _ffi
from prana_b200 import kernels as K

pytestmark = pytest.mark.gpu

TOL = 2e-5  # same kernels as the allocating entry point; normwise relative


def _setup(nh, nkv, hd, pos, seed):
    rng = np.random.default_rng(seed)
    kc = torch.from_numpy(rng.standard_normal((pos + 1, nkv * hd)).astype(np.float16).view(np.int16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((pos + 1, nkv * hd)).astype(np.float16).view(np.int16)).cuda()
    q = torch.from_numpy(rng.standard_normal(nh * hd).astype(np.float32)).cuda()
    return q, kc, vc


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("nh,nkv,hd,pos", [(32, 8, 128, 4095), (14, 2, 64, 700), (6, 6, 48, 255), (8, 1, 64, 5)])
def test_noalloc_matches_allocating_entry_point(gpu, nh, nkv, hd, pos):
    q, kc, vc = _setup(nh, nkv, hd, pos, seed=11)
    ref = K.attention_decode(q, kc, vc, pos, nh, nkv, hd)
    out = torch.empty_like(ref)
    for _ in range(2):
        out.fill_(float("nan"))
        got = K.attention_decode_noalloc(q, kc, vc, pos, nh, nkv, hd, out=out)
        torch.cuda.synchronize()
        assert rel(got, ref) < TOL


def test_noalloc_rejects_shapes_beyond_the_static_scratch(gpu):
    # 8 kv heads x 32 splits x 32 query heads each x (128 + 2) floats > 1,048,576
    nh, nkv, hd, pos = 256, 8, 128, 4095
    q, kc, vc = _setup(nh, nkv, hd, pos, seed=12)
    with pytest.raises(_ffi.PranaError, match="static scratch holds"):
        K.attention_decode_noalloc(q, kc, vc, pos, nh, nkv, hd)
    # the allocating entry point still serves the shape
    out = K.attention_decode(q, kc, vc, pos, nh, nkv, hd)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
