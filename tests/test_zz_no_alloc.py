"""GPU check of vlak_attn_gqa_fwd_noalloc, the entry point that allocates
nothing (its key-split scratch is the library's static device buffer).

Through the C ABI, two calls in a row on a small batch (C3 at B = 1, which
splits its keys and so uses the scratch) must each match the existing
workspace entry point, vlak_attn_gqa_fwd_ws, within the kernel tests'
tolerance (atol 1e-2, rtol 1.6e-2). A problem whose scratch would exceed the
static buffer is rejected before anything is launched.
"""
import ctypes

import pytest
import torch

from tests import capi

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 1.6e-2


def _noalloc(q, k, v, o, prefix_len):
    L = capi.lib()
    L.vlak_attn_gqa_fwd_noalloc.argtypes = [ctypes.POINTER(capi.GqaArgs), ctypes.c_void_p]
    a = capi.gqa_args(q, k, v, o, prefix_len=prefix_len)
    return L.vlak_attn_gqa_fwd_noalloc(ctypes.byref(a), capi.stream_ptr())


def test_noalloc_matches_workspace_entry_point_twice():
    g = torch.Generator(device="cuda").manual_seed(31)
    q = torch.randn(1, 50, 15, 64, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(1, 291, 5, 64, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(1, 291, 5, 64, device="cuda", generator=g).to(torch.bfloat16)
    assert capi.workspace_size(q, k, v, prefix_len=241) > 0  # the split (scratch) path runs
    for _ in range(2):
        o = torch.empty_like(q)
        st = _noalloc(q, k, v, o, 241)
        assert st == capi.VLAK_OK, capi.last_error()
        st, ref = capi.attn_gqa_ws(q, k, v, prefix_len=241)
        assert st == capi.VLAK_OK, capi.last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_noalloc_rejects_a_problem_beyond_its_scratch():
    # SigLIP-sized self-attention: 1 x 1024 queries x 12 heads would split
    # into about 10 MB of scratch, more than the 8 MiB buffer
    q = torch.zeros(1, 1024, 12, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 1024, 12, 64, device="cuda", dtype=torch.bfloat16)
    assert capi.workspace_size(q, k, k, prefix_len=-1) > (8 << 20)
    o = torch.empty_like(q)
    st = _noalloc(q, k, k, o, -1)
    assert st == capi.VLAK_ERR_INVALID_ARGUMENT
    assert "static buffer" in capi.last_error()
