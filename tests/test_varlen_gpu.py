"""GPU parity of vlak::fused_attention_gqa_varlen (per-sample lengths, the C4
prefix site) against the CPU oracle and the ref_sdpa golden vectors.

visible(r, c) = c < L_b and r < L_b; rows r >= L_b are exact zeros.
Tolerance: bf16 output vs the float64 oracle, atol 1e-2 / rtol 1.6e-2.
"""
import os

import numpy as np
import pytest
import torch

from oracle import gqa_attention_varlen
from tests.golden.make_golden import VARLEN_CASES, attn_inputs
from tests.test_attention_gpu import check, device_error

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def varlen(*a, **kw):
    from kernels.attention import fused_attention_gqa_varlen
    return fused_attention_gqa_varlen(*a, **kw)


def inputs(B, M, N, H, Hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).bfloat16()  # noqa: E731
    return mk(B, M, H, 64), mk(B, N, Hkv, 64), mk(B, N, Hkv, 64)


def oracle(q, k, v, lengths, scale=None):
    return torch.from_numpy(gqa_attention_varlen(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                 v.float().cpu().numpy(),
                                                 lengths.cpu().numpy(), scale))


def c4_lengths(B, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(150, 242, (B,), generator=g)


@pytest.mark.parametrize("idx", range(len(VARLEN_CASES)))
def test_golden_ref_sdpa(idx):
    g = np.load(os.path.join(GOLDEN, "varlen_golden.npz"))
    B, M, N, H, Hkv, lengths, seed = VARLEN_CASES[idx]
    q, k, v = (t.cuda() for t in attn_inputs(B, M, N, H, Hkv, seed))
    L = torch.tensor(lengths, device="cuda")
    ref = torch.from_numpy(np.nan_to_num(g[f"v{idx}__out"].astype(np.float64), nan=0.0))
    check(varlen(q, k, v, L), ref)


@pytest.mark.parametrize("B", [1, 16])
def test_c4_prefix_shapes(B):
    q, k, v = inputs(B, 241, 241, 15, 5, B)
    L = c4_lengths(B, B).cuda()
    out = varlen(q, k, v, L)
    assert out.shape == q.shape and out.is_contiguous()
    check(out, oracle(q, k, v, L))


def test_c4_batch128_sampled():
    B = 128
    q, k, v = inputs(B, 241, 241, 15, 5, 128)
    L = c4_lengths(B, 128).cuda()
    out = varlen(q, k, v, L)
    idx = torch.tensor([0, 1, 63, 127], device="cuda")
    check(out[idx], oracle(q[idx], k[idx], v[idx], L[idx]))


def test_compacted_197_all_visible_equals_unmasked():
    # the compacted variant M = N = 197 with L = 197: every pair visible, the
    # same result as the analytic op with no mask, bit for bit
    from kernels.attention import fused_attention_gqa
    q, k, v = inputs(4, 197, 197, 15, 5, 11)
    L = torch.full((4,), 197, device="cuda")
    a = varlen(q, k, v, L)
    b = fused_attention_gqa(q, k, v)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    check(a, oracle(q, k, v, L))


@pytest.mark.parametrize("lengths", [(0, 0), (1, 241), (241, 0), (300, -5), (64, 65), (128, 129)])
def test_edge_lengths(lengths):
    B = len(lengths)
    q, k, v = inputs(B, 241, 241, 6, 2, 3)
    L = torch.tensor(lengths, device="cuda")
    out = varlen(q, k, v, L)
    for b, Lb in enumerate(lengths):
        Lc = min(max(Lb, 0), 241)
        assert (out[b, Lc:] == 0).all()
    check(out, oracle(q, k, v, L))


def test_int32_and_int64_lengths_agree():
    q, k, v = inputs(3, 241, 241, 15, 5, 4)
    L = c4_lengths(3, 4)
    a = varlen(q, k, v, L.cuda().to(torch.int64))
    b = varlen(q, k, v, L.cuda().to(torch.int32))
    torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_strided_views():
    # q/k/v as slices of a fused projection, read in place
    B, M, H, Hkv = 2, 241, 15, 5
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(B, M, H + 2 * Hkv, 64, device="cuda", generator=g).bfloat16()
    q, k, v = qkv[:, :, :H], qkv[:, :, H:H + Hkv], qkv[:, :, H + Hkv:]
    L = torch.tensor([200, 241], device="cuda")
    check(varlen(q, k, v, L), oracle(q, k, v, L))


def test_cuda_graph_capture():
    q, k, v = inputs(2, 241, 241, 15, 5, 6)
    L = torch.tensor([170, 230], device="cuda")
    ref = varlen(q, k, v, L)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        varlen(q, k, v, L)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = varlen(q, k, v, L)
    graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    assert device_error() == 0


@pytest.mark.parametrize("bad", ["cpu_lengths", "float_lengths", "short_lengths", "fp32_q"])
def test_bad_inputs_raise(bad):
    q, k, v = inputs(2, 16, 16, 2, 1, 7)
    L = torch.tensor([8, 16], device="cuda")
    if bad == "cpu_lengths":
        L = L.cpu()
    elif bad == "float_lengths":
        L = L.float()
    elif bad == "short_lengths":
        L = L[:1]
    elif bad == "fp32_q":
        q = q.float()
    with pytest.raises(RuntimeError):
        varlen(q, k, v, L)
