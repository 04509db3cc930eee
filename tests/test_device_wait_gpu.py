"""Failure path of the bounded device waits, without a GPU fault.

A kernel waits on a barrier that nothing completes; after the 1 s limit it must
record VLAK_ERR_DEVICE_TIMEOUT in the device error word and return, and the
context must stay usable: the next attention call runs and matches the oracle.
"""
import ctypes

import pytest
import torch

from tests import capi
from tests.test_attention_gpu import check, device_error, oracle, rand

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_survives():
    assert device_error() == 0
    L = capi.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.vlak_selftest_wait_timeout(st) == capi.VLAK_OK
    torch.cuda.synchronize()  # the kernel returns after its wait limit
    assert device_error() == capi.VLAK_ERR_DEVICE_TIMEOUT
    assert device_error() == 0  # reading clears the word

    from kernels.attention import fused_attention_gqa_v4
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = rand(2, 50, 15, 64, gen=g), rand(2, 291, 5, 64, gen=g), rand(2, 291, 5, 64, gen=g)
    out = fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=241)
    check(out, oracle(q, k, v, 241, 0, 0, 0.125))
