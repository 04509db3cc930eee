"""GPU parity of vlak::fused_attention, the (B, H, M, 64) op with a bool or
analytic mask (kernels/attention/fused_attention.cu:525-598), against the CPU
oracle and the ref_sdpa golden vectors. Mirrors tests/test_attention.py of the
reference: its shape grid, masks, custom scale, extreme values, the analytic ==
tensor-mask identity and torch.compile.

Tolerances (output vs the float64 oracle): fp32 2e-5, fp16 2e-3 (the
reference's), bf16 atol 1e-2 / rtol 1.6e-2 (tighter than
the reference's 2e-2). Rows with no visible key are exact zeros.
"""
import os

import numpy as np
import pytest
import torch

from oracle import sdpa_bhmd
from tests.golden.make_golden import SDPA_CASES, bhmd_inputs, smolvla_pattern
from tests.test_attention_gpu import device_error

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = {torch.float32: (2e-5, 2e-5), torch.float16: (2e-3, 2e-3), torch.bfloat16: (1.6e-2, 1e-2),
       torch.float64: (2e-5, 2e-5)}

# tests/test_attention.py:13-20
SHAPES = [(1, 15, 50, 291), (1, 15, 50, 241), (1, 15, 241, 241), (1, 12, 1024, 1024),
          (1, 1, 1, 1), (2, 3, 17, 33)]


def fa(*args, **kw):
    from kernels.attention import fused_attention
    return fused_attention(*args, **kw)


def inputs(B, H, M, N, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(dtype)  # noqa: E731
    return mk(B, H, M, 64), mk(B, H, N, 64), mk(B, H, N, 64)


def oracle(q, k, v, mask=None, prefix_len=None, scale=None):
    m = mask.cpu().numpy() if mask is not None else None
    return torch.from_numpy(sdpa_bhmd(q.double().cpu().numpy(), k.double().cpu().numpy(),
                                      v.double().cpu().numpy(), attn_mask=m,
                                      prefix_len=prefix_len, scale=scale))


def check(out, ref, dtype):
    torch.cuda.synchronize()
    assert device_error() == 0
    got = out.double().cpu()
    zero = (ref == 0).all(dim=-1)
    assert (got[zero] == 0).all(), "rows with no visible key must be exact zeros"
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(got, ref, rtol=rtol, atol=atol)


def pattern(B, M, N, prefix):
    return smolvla_pattern(M, N, prefix)[None].expand(B, M, N).contiguous().cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
def test_unmasked_matches_oracle(dtype, shape):
    B, H, M, N = shape
    q, k, v = inputs(B, H, M, N, dtype, 0)
    out = fa(q, k, v)
    assert out.shape == q.shape and out.dtype == dtype and out.is_contiguous()
    if M * N > 300_000:  # check a slice of heads at the vision size
        check(out[:, :2], oracle(q[:, :2], k[:, :2], v[:, :2]), dtype)
    else:
        check(out, oracle(q, k, v), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape,prefix", [((1, 15, 50, 291), 241), ((1, 15, 50, 241), 191),
                                          ((1, 15, 241, 241), 241), ((2, 4, 33, 65), 32)])
def test_masked_matches_oracle(dtype, shape, prefix):
    B, H, M, N = shape
    q, k, v = inputs(B, H, M, N, dtype, 5)
    mask = pattern(B, M, N, prefix)
    check(fa(q, k, v, attn_mask=mask), oracle(q, k, v, mask=mask), dtype)


@pytest.mark.parametrize("shape,prefix", [((1, 15, 50, 291), 241), ((1, 15, 50, 241), 191),
                                          ((1, 15, 241, 241), 241), ((2, 4, 33, 65), 32)])
def test_analytic_mask_equals_tensor_mask(shape, prefix):
    # tests/test_attention.py:85-105: the two routes are bit-identical
    B, H, M, N = shape
    q, k, v = inputs(B, H, M, N, torch.bfloat16, 9)
    mask = pattern(B, M, N, prefix)
    a = fa(q, k, v, prefix_len=prefix)
    b = fa(q, k, v, attn_mask=mask)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    check(a, oracle(q, k, v, mask=mask), torch.bfloat16)


@pytest.mark.parametrize("idx", range(len(SDPA_CASES)))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_golden_ref_sdpa(idx, dtype):
    g = np.load(os.path.join(GOLDEN, "sdpa_golden.npz"))
    B, H, M, N, kind, seed = SDPA_CASES[idx]
    q, k, v = (t.to(dtype).cuda() for t in bhmd_inputs(B, H, M, N, seed))
    mask = None
    if f"s{idx}__mask" in g:
        bits = np.unpackbits(g[f"s{idx}__mask"])[: B * M * N].reshape(B, M, N).astype(bool)
        mask = torch.from_numpy(bits).cuda()
    ref = torch.from_numpy(np.nan_to_num(g[f"s{idx}__out"].astype(np.float64), nan=0.0))
    check(fa(q, k, v, attn_mask=mask), ref, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fully_masked_rows_are_zero(dtype):
    B, H, M, N = 2, 3, 40, 70
    q, k, v = inputs(B, H, M, N, dtype, 4)
    mask = torch.rand(B, M, N, device="cuda") < 0.5
    mask[0, :7] = False
    mask[1, 39] = False
    out = fa(q, k, v, attn_mask=mask)
    assert (out[0, :, :7] == 0).all() and (out[1, :, 39] == 0).all()
    check(out, oracle(q, k, v, mask=mask), dtype)


def test_custom_scale():
    q, k, v = inputs(1, 2, 8, 16, torch.float32, 2)
    check(fa(q, k, v, scale=0.5), oracle(q, k, v, scale=0.5), torch.float32)
    qb, kb, vb = (t.bfloat16() for t in (q, k, v))
    check(fa(qb, kb, vb, scale=0.3), oracle(qb, kb, vb, scale=0.3), torch.bfloat16)


def test_matches_torch_sdpa_fp32():
    import torch.nn.functional as F
    q, k, v = inputs(1, 15, 50, 291, torch.float32, 1)
    torch.testing.assert_close(fa(q, k, v), F.scaled_dot_product_attention(q, k, v),
                               rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_extreme_values_stable(dtype):
    q = torch.full((1, 1, 4, 64), 30.0, device="cuda", dtype=dtype)
    k = torch.full((1, 1, 8, 64), 30.0, device="cuda", dtype=dtype)
    v = torch.randn(1, 1, 8, 64, device="cuda").to(dtype)
    out = fa(q, k, v)
    assert torch.isfinite(out).all()
    check(out, oracle(q, k, v), dtype)


def test_noncontiguous_inputs_are_accepted():
    q, k, v = inputs(2, 3, 20, 40, torch.bfloat16, 3)
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)  # same values, other strides
    check(fa(qt, k, v), oracle(q, k, v), torch.bfloat16)


def test_fp64_runs_in_fp32_math():
    q, k, v = inputs(1, 2, 9, 20, torch.float64, 6)
    out = fa(q, k, v)
    assert out.dtype == torch.float64
    check(out, oracle(q, k, v), torch.float64)


def test_composes_with_torch_compile():
    q, k, v = inputs(1, 15, 50, 291, torch.bfloat16, 7)
    mask = pattern(1, 50, 291, 241)

    def f(q, k, v):
        return fa(q, k, v, attn_mask=mask) * 2

    eager = f(q, k, v)
    compiled = torch.compile(f, fullgraph=True)(q, k, v)
    torch.testing.assert_close(compiled, eager, rtol=0, atol=0)


@pytest.mark.parametrize("bad", ["dims", "head_dim", "mask_dtype", "mask_shape", "prefix_fp32",
                                 "kv_len", "heads"])
def test_bad_inputs_raise(bad):
    q, k, v = inputs(1, 2, 8, 16, torch.float32, 8)
    mask = torch.ones(1, 8, 16, dtype=torch.bool, device="cuda")
    kw = {}
    if bad == "dims":
        q = q[0]
    elif bad == "head_dim":
        q = q[..., :32]
    elif bad == "mask_dtype":
        kw["attn_mask"] = mask.float()
    elif bad == "mask_shape":
        kw["attn_mask"] = mask[:, :4]
    elif bad == "prefix_fp32":
        kw["prefix_len"] = 4
    elif bad == "kv_len":
        v = v[:, :, :8]
    elif bad == "heads":
        k = k[:, :1]
    with pytest.raises(RuntimeError):
        fa(q, k, v, **kw)
