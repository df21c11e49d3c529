"""Bounded device waits that run out (GPU, no fault).

Every spin in the library's kernels is bounded; when the awaited data never
arrives the kernel raises the device error word and returns, and the host
turns it into PRANA_E_TIMEOUT on the next synchronization.  These tests make
two kinds of wait run out on data nothing writes -- an mbarrier no copy
completes, and the peer exchange's receive wait with a rank that never stores
(both receive areas on this one GPU) -- and check that the status comes back
and the context keeps working afterwards.
"""
import pytest
import torch

from prana_b200 import _ffi
from prana_b200 import kernels as K

pytestmark = pytest.mark.gpu

TIMEOUT = -6  # PRANA_E_TIMEOUT


@pytest.mark.parametrize("which,polls", [(0, 1 << 12), (1, 1 << 12)])
def test_wait_runs_out_and_context_stays_usable(gpu, which, polls):
    assert K.debug_wait_timeout(which, polls) == TIMEOUT
    # reported once: the next synchronization is clean
    K.synchronize()
    # the context still computes
    x = torch.randn(3, 64, device="cuda")
    acts = K.quantize_acts(x)
    K.synchronize()
    assert acts.q.shape == (3, 64)
    # and a second timeout is reported again
    assert K.debug_wait_timeout(which, polls) == TIMEOUT


def test_noalloc_call_leaves_no_error(gpu):
    nh, nkv, hd, pos = 8, 2, 64, 300
    kc = torch.randn(pos + 1, nkv * hd, device="cuda").half().view(torch.int16)
    vc = torch.randn(pos + 1, nkv * hd, device="cuda").half().view(torch.int16)
    q = torch.randn(nh * hd, device="cuda")
    K.attention_decode_noalloc(q, kc, vc, pos, nh, nkv, hd)
    K.synchronize()  # healthy copies: no timeout reported


def test_bad_selector_is_invalid(gpu):
    with pytest.raises(_ffi.PranaError, match="PRANA_E_INVALID"):
        _ffi.call("prana_debug_wait_timeout", K.context(), 7, 1)
