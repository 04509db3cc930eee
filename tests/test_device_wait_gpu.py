"""Failure path of the bounded device waits, without a GPU fault.

A kernel waits on a barrier that nothing completes; after the 1 s limit it must
record VLAK_ERR_DEVICE_TIMEOUT and return, and the context must stay usable:
the next attention call runs and matches the oracle. The torch ops must raise
the recorded status as RuntimeError on their next call (read from the
host-mapped error word, no device synchronization), and the synchronous
vlak::device_error op must return it.
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


def _inputs(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return rand(2, 50, 15, 64, gen=g), rand(2, 291, 5, 64, gen=g), rand(2, 291, 5, 64, gen=g)


def _selftest():
    L = capi.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.vlak_selftest_wait_timeout(st) == capi.VLAK_OK


def test_expired_wait_raises_in_the_next_torch_op():
    from kernels.attention import fused_attention_gqa_v4
    from kernels.softmax import softmax

    q, k, v = _inputs(4)
    fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=241)  # sets up the host word
    torch.cuda.synchronize()
    assert device_error() == 0
    _selftest()
    torch.cuda.synchronize()  # the self-test kernel has given up its wait
    with pytest.raises(RuntimeError, match="bounded device wait"):
        fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=241)
    # the read cleared the word: the next call runs and is correct
    out = fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=241)
    check(out, oracle(q, k, v, 241, 0, 0, 0.125))
    # the softmax op checks the word as well
    _selftest()
    torch.cuda.synchronize()
    x = torch.randn(64, 1024, device="cuda")
    with pytest.raises(RuntimeError, match="bounded device wait"):
        softmax(x)
    torch.testing.assert_close(softmax(x), torch.softmax(x, dim=-1), rtol=1e-5, atol=1e-6)


def test_device_error_op_is_synchronous():
    from kernels.attention import check_device_error, device_error as op_error

    assert op_error() == 0
    _selftest()  # no synchronize: the op waits for the device itself
    assert op_error() == capi.VLAK_ERR_DEVICE_TIMEOUT
    assert op_error() == 0
    check_device_error()
    _selftest()
    with pytest.raises(RuntimeError, match="bounded device wait"):
        check_device_error()
    assert device_error() == 0


def test_poll_reads_the_host_word_without_synchronizing():
    L = capi.lib()
    code = ctypes.c_int(-1)
    assert L.vlak_device_error_poll(ctypes.byref(code)) == capi.VLAK_OK
    assert code.value == 0
    _selftest()
    torch.cuda.synchronize()
    assert L.vlak_device_error_poll(ctypes.byref(code)) == capi.VLAK_OK
    assert code.value == capi.VLAK_ERR_DEVICE_TIMEOUT
    assert L.vlak_device_error_poll(ctypes.byref(code)) == capi.VLAK_OK
    assert code.value == 0
    assert device_error() == 0
