"""GPU parity of vlak::fused_attention_gqa / _v4 (the tcgen05 kernel) against
the CPU oracle, on the reference's case grid (tests/test_attention_gqa.py:43-54),
the golden vectors, the benchmark configurations and edge cases.

Tolerance: atol 1e-2, rtol 1.6e-2 against the float64 oracle, plus the
reference's own gate (cosine > 0.999, max_abs < 3e-2); rows with no visible
key must be exact zeros.
"""
import os

import numpy as np
import pytest
import torch

from kernels import workloads as wl
from kernels.attention import fused_attention_gqa, fused_attention_gqa_v4
from oracle import gqa_attention
from tests import capi
from tests.golden.make_golden import ATTN_CASES, attn_inputs as golden_inputs

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 1.6e-2

# (B, M, N, H, Hkv, P, ds, de): tests/test_attention_gqa.py:43-54
CASES = [
    (1, 50, 241, 15, 5, 241, 196, 240),
    (1, 50, 291, 15, 5, 241, 196, 240),
    (1, 50, 241, 15, 5, 241, 0, 0),
    (2, 37, 127, 8, 8, 100, 20, 44),
    (1, 100, 256, 12, 4, 200, 64, 96),
    (1, 32, 64, 4, 2, 64, 0, 0),
    (1, 33, 65, 4, 2, 40, 8, 16),
    (3, 50, 241, 15, 5, 241, 196, 240),
    (1, 40, 128, 6, 2, 128, 32, 64),
    (1, 50, 241, 15, 5, 241, 200, 232),
]
# shapes beyond the reference grid: tiny / wide / many heads per group /
# multi-chunk / multi-block query ranges
EXTRA = [
    (1, 1, 1, 1, 1, 1, 0, 0),
    (1, 1, 300, 2, 1, 300, 0, 0),
    (2, 5, 17, 16, 1, 9, 2, 5),
    (1, 241, 241, 15, 5, 241, 0, 0),
    (2, 197, 197, 15, 5, 197, 0, 0),
    (1, 300, 700, 4, 4, 600, 100, 300),
    (1, 64, 1024, 12, 12, 1024, 0, 0),
    (1, 20, 40, 128, 1, 40, 0, 0),
    (4, 50, 291, 15, 5, 241, 0, 0),
    (1, 8, 256, 1, 1, 256, 0, 0),
    (3, 8, 300, 1, 1, 300, 0, 0),
    (2, 16, 1000, 2, 1, 1000, 300, 700),
]


def rand(*shape, gen):
    return torch.randn(*shape, device="cuda", generator=gen).to(torch.bfloat16)


def oracle(q, k, v, P, ds, de, scale=None):
    return torch.from_numpy(gqa_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                          v.float().cpu().numpy(), P, ds, de, scale))


def device_error() -> int:
    import ctypes
    code = ctypes.c_int(-1)
    assert capi.lib().vlak_device_error_read(ctypes.byref(code)) == capi.VLAK_OK
    return code.value


def check(out, ref, P=None):
    torch.cuda.synchronize()
    assert device_error() == 0, "a bounded device wait expired inside the kernel"
    got = out.float().cpu().double()
    zero_rows = (ref == 0).all(dim=-1)
    assert (got[zero_rows] == 0).all(), "rows with no visible key must be exact zeros"
    torch.testing.assert_close(got, ref, atol=ATOL, rtol=RTOL)
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    if ref.abs().max() > 0:
        assert cos > 0.999 and (got - ref).abs().max().item() < 3e-2


def run(fn, B, M, N, H, Hkv, P, ds, de, seed=0, scale=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = rand(B, M, H, 64, gen=g), rand(B, N, Hkv, 64, gen=g), rand(B, N, Hkv, 64, gen=g)
    out = fn(q, k, v, scale=scale, prefix_len=P, dead_start=ds, dead_end=de)
    assert out.shape == (B, M, H, 64) and out.is_contiguous() and out.dtype == torch.bfloat16
    check(out, oracle(q, k, v, P, ds, de, scale))
    return out


@pytest.mark.parametrize("fn", [fused_attention_gqa, fused_attention_gqa_v4])
@pytest.mark.parametrize("case", CASES + EXTRA)
def test_parity(fn, case):
    run(fn, *case)


@pytest.mark.parametrize("idx", range(len(ATTN_CASES)))
def test_golden_vectors(idx):
    B, M, N, H, Hkv, P, ds, de, seed = ATTN_CASES[idx]
    q, k, v = (t.cuda() for t in golden_inputs(B, M, N, H, Hkv, seed))
    ref = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))[f"c{idx}__out"]
    ref = torch.from_numpy(ref).double()
    out = fused_attention_gqa(q, k, v, prefix_len=P, dead_start=ds, dead_end=de).float().cpu().double()
    nan_rows = torch.isnan(ref).all(-1)
    assert (out[nan_rows] == 0).all()
    torch.testing.assert_close(out[~nan_rows], ref[~nan_rows], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_c3_expert_self_attention(B):
    s = wl.expert_shape(B)
    q, k, v = wl.attn_inputs(s, seed=B)
    out = fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=s.P)
    check(out, oracle(q, k, v, s.P, 0, 0, 0.125))


@pytest.mark.parametrize("B", [1, 16])
def test_c4_prefix_bidirectional(B):
    s = wl.AttnShape(B=B, M=241, N=241, H=15, Hkv=5, P=241)
    q, k, v = wl.attn_inputs(s, seed=7)
    check(fused_attention_gqa(q, k, v), oracle(q, k, v, 241, 0, 0))


def test_c5_batch_2048_properties():
    s = wl.expert_shape(2048)
    q, k, v = wl.attn_inputs(s, seed=11)
    a = fused_attention_gqa_v4(q, k, v, prefix_len=s.P)
    b = fused_attention_gqa_v4(q, k, v, prefix_len=s.P)
    assert torch.equal(a, b)                              # deterministic
    assert torch.isfinite(a.float()).all()
    idx = torch.tensor([0, 1, 511, 1024, 1777, 2047])
    check(a[idx.cuda()], oracle(q[idx.cuda()], k[idx.cuda()], v[idx.cuda()], s.P, 0, 0))


# Shapes with one query block whose second M-tile holds at most 32 rows (the
# kernel's narrow warp layout), over several GQA ratios, masks and batches
# (the small batches also take the key-split path):
# (B, M, N, H, Hkv, P, ds, de)
NARROW = [
    (2, 150, 300, 4, 4, 250, 0, 0),      # G=1: 22 rows in tile 1
    (1, 70, 200, 8, 4, 150, 20, 60),     # G=2: 12 rows
    (3, 38, 100, 16, 4, 100, 0, 0),      # G=4: 24 rows
    (1, 19, 77, 8, 1, 50, 10, 20),       # G=8: 24 rows
    (2, 30, 64, 5, 1, 64, 0, 0),         # G=5: 25 rows
    (96, 50, 291, 15, 5, 241, 196, 240),  # C3 with the real dead band, unsplit
    (2, 43, 100, 15, 5, 80, 0, 0),       # G=3: tile 1 holds one position (3 rows)
    (2, 52, 291, 15, 5, 241, 196, 240),  # G=3: 10 positions, 30 rows (the most for G=3)
    (1, 10, 130, 16, 1, 100, 30, 70),    # G=16: 2 positions, exactly 32 rows
    (3, 160, 161, 2, 2, 161, 0, 0),      # G=1: 32 rows, a one-key last chunk
]


@pytest.mark.parametrize("case", NARROW)
def test_narrow_layout_shapes(case):
    run(fused_attention_gqa, *case, seed=12)


def test_strided_inputs():
    # tests/test_attention_gqa.py:66-74
    g = torch.Generator(device="cuda").manual_seed(1)
    qb, kb, vb = rand(1, 50, 17, 64, gen=g), rand(1, 241, 7, 64, gen=g), rand(1, 241, 7, 64, gen=g)
    q, k, v = qb[:, :, 1:16], kb[:, :, 1:6], vb[:, :, 2:7]
    assert not q.is_contiguous()
    for fn in (fused_attention_gqa, fused_attention_gqa_v4):
        check(fn(q, k, v, prefix_len=241, dead_start=196, dead_end=240),
              oracle(q, k, v, 241, 196, 240))


def test_transposed_query_layout():
    # (B, H, M, D) storage viewed as (B, M, H, D), as the stress test of the reference does
    g = torch.Generator(device="cuda").manual_seed(2)
    q = rand(2, 15, 50, 64, gen=g).transpose(1, 2)
    k, v = rand(2, 291, 5, 64, gen=g), rand(2, 291, 5, 64, gen=g)
    check(fused_attention_gqa(q, k, v, prefix_len=241, dead_start=196, dead_end=240),
          oracle(q, k, v, 241, 196, 240))


def test_matches_sdpa_unmasked():
    g = torch.Generator(device="cuda").manual_seed(2)
    q, k, v = rand(1, 50, 15, 64, gen=g), rand(1, 241, 5, 64, gen=g), rand(1, 241, 5, 64, gen=g)
    out = fused_attention_gqa(q, k, v, prefix_len=241).float()
    ke, ve = k.repeat_interleave(3, dim=2), v.repeat_interleave(3, dim=2)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2).float(), ke.transpose(1, 2).float(), ve.transpose(1, 2).float()
    ).transpose(1, 2)
    torch.testing.assert_close(out, ref, rtol=RTOL, atol=ATOL)


def test_custom_scale():
    run(fused_attention_gqa, 1, 8, 16, 2, 2, 16, 0, 0, scale=0.5)


def test_extreme_logits_stay_finite():
    q = torch.full((1, 4, 1, 64), 30.0, device="cuda", dtype=torch.bfloat16)
    k = torch.full((1, 8, 1, 64), 30.0, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, 8, 1, 64, device="cuda").to(torch.bfloat16)
    out = fused_attention_gqa(q, k, v)
    assert torch.isfinite(out.float()).all()
    check(out, oracle(q, k, v, 8, 0, 0))


def test_large_score_growth_across_chunks_rescales():
    # the second key chunk holds far larger scores than the first: the lazily
    # updated row max must move and rescale O and l
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.ones(1, 4, 2, 64, device="cuda", dtype=torch.bfloat16) * 0.5
    k = rand(1, 300, 1, 64, gen=g) * 0.1
    k[:, 128:256] += 2.0
    v = rand(1, 300, 1, 64, gen=g)
    check(fused_attention_gqa(q, k, v), oracle(q, k, v, 300, 0, 0))


def test_fully_masked_rows_are_exact_zeros():
    # rows 0..7 see no key: prefix entirely dead, staircase starts at row 8
    g = torch.Generator(device="cuda").manual_seed(6)
    q, k, v = rand(2, 12, 4, 64, gen=g), rand(2, 16, 2, 64, gen=g), rand(2, 16, 2, 64, gen=g)
    for fn in (fused_attention_gqa, fused_attention_gqa_v4):
        out = fn(q, k, v, prefix_len=12, dead_start=0, dead_end=12)
        assert (out[:, :8] == 0).all()
        assert (out[:, 8:].float().abs().sum(-1) > 0).all()


def test_empty_and_zero_key_problems():
    z = torch.empty(0, 5, 3, 64, device="cuda", dtype=torch.bfloat16)
    kz = torch.empty(0, 7, 1, 64, device="cuda", dtype=torch.bfloat16)
    assert fused_attention_gqa(z, kz, kz).shape == (0, 5, 3, 64)
    q = torch.randn(2, 3, 4, 64, device="cuda").to(torch.bfloat16)
    k0 = torch.empty(2, 0, 2, 64, device="cuda", dtype=torch.bfloat16)
    out = fused_attention_gqa(q, k0, k0)
    assert out.shape == (2, 3, 4, 64) and (out == 0).all()


def test_v4_equals_v3():
    g = torch.Generator(device="cuda").manual_seed(2)
    for N in (241, 291):
        q, k, v = rand(1, 50, 15, 64, gen=g), rand(1, N, 5, 64, gen=g), rand(1, N, 5, 64, gen=g)
        a = fused_attention_gqa(q, k, v, prefix_len=241, dead_start=196, dead_end=240)
        b = fused_attention_gqa_v4(q, k, v, prefix_len=241, dead_start=196, dead_end=240)
        assert torch.equal(a, b)


@pytest.mark.parametrize("fn", [fused_attention_gqa, fused_attention_gqa_v4])
def test_composes_with_torch_compile(fn):
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = rand(1, 50, 15, 64, gen=g), rand(1, 241, 5, 64, gen=g), rand(1, 241, 5, 64, gen=g)
    eager = fn(q, k, v, prefix_len=241, dead_start=196, dead_end=240)

    @torch.compile(fullgraph=True)
    def f(q, k, v):
        return fn(q, k, v, prefix_len=241, dead_start=196, dead_end=240)

    assert torch.equal(f(q, k, v), eager)


def test_cuda_graph_capture_replays():
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = rand(8, 50, 15, 64, gen=g), rand(8, 291, 5, 64, gen=g), rand(8, 291, 5, 64, gen=g)
    eager = fused_attention_gqa(q, k, v, prefix_len=241)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fused_attention_gqa(q, k, v, prefix_len=241)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fused_attention_gqa(q, k, v, prefix_len=241)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # B = 8 runs the key-split form: the captured workspace and merge must
    # serve new inputs on replay
    for seed in (5, 6):
        g2 = torch.Generator(device="cuda").manual_seed(seed)
        q.copy_(rand(8, 50, 15, 64, gen=g2))
        k.copy_(rand(8, 291, 5, 64, gen=g2))
        v.copy_(rand(8, 291, 5, 64, gen=g2))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, fused_attention_gqa(q, k, v, prefix_len=241))


def test_stress_randomized():
    # tests/test_attention_gqa.py:107-131: allocator churn, every trial checked
    fails = []
    for trial in range(30):
        g = torch.Generator(device="cuda").manual_seed(100 + trial)
        N = 241 if trial % 2 == 0 else 291
        q = rand(1, 15, 50, 64, gen=g).transpose(1, 2)
        k, v = rand(1, N, 5, 64, gen=g), rand(1, N, 5, 64, gen=g)
        junk = [torch.empty(int(torch.randint(1000, 200000, (1,)).item()), device="cuda",
                            dtype=torch.bfloat16) for _ in range(4)]
        for _ in range(10):
            out = fused_attention_gqa(q, k, v, prefix_len=241, dead_start=196, dead_end=240)
        del junk
        ref = oracle(q, k, v, 241, 196, 240)
        assert device_error() == 0
        cos = torch.nn.functional.cosine_similarity(out.float().cpu().double().flatten(),
                                                    ref.flatten(), dim=0).item()
        if cos < 0.999:
            fails.append((trial, cos))
    assert not fails, f"corrupted trials: {fails}"


def test_rejects_bad_inputs():
    # tests/test_attention_gqa.py:134-143
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = rand(1, 50, 15, 64, gen=g), rand(1, 241, 5, 64, gen=g), rand(1, 241, 5, 64, gen=g)
    with pytest.raises(RuntimeError):
        fused_attention_gqa(q.float(), k.float(), v.float())
    with pytest.raises(RuntimeError):
        fused_attention_gqa(q, k, v, prefix_len=100, dead_start=90, dead_end=120)
    with pytest.raises(RuntimeError):
        fused_attention_gqa(q, rand(1, 241, 4, 64, gen=g), rand(1, 241, 4, 64, gen=g))
    with pytest.raises(RuntimeError):
        fused_attention_gqa_v4(q[..., :32], k[..., :32], v[..., :32])
    with pytest.raises(RuntimeError):
        fused_attention_gqa(q, k, v, prefix_len=300)


@pytest.mark.parametrize("v4", [False, True])
def test_through_c_abi(v4):
    g = torch.Generator(device="cuda").manual_seed(9)
    q, k, v = rand(3, 50, 15, 64, gen=g), rand(3, 291, 5, 64, gen=g), rand(3, 291, 5, 64, gen=g)
    st, o = capi.attn_gqa(q, k, v, prefix_len=241, dead_start=196, dead_end=240, v4=v4)
    assert st == capi.VLAK_OK, capi.last_error()
    torch.cuda.synchronize()
    check(o, oracle(q, k, v, 241, 196, 240))
    # the torch op runs the key-split form at this small batch: same result
    # through the C ABI's workspace entry point
    st, o_ws = capi.attn_gqa_ws(q, k, v, prefix_len=241, dead_start=196, dead_end=240)
    assert st == capi.VLAK_OK, capi.last_error()
    assert torch.equal(o_ws, fused_attention_gqa(q, k, v, prefix_len=241, dead_start=196, dead_end=240))


def test_device_error_word_stays_clear():
    run(fused_attention_gqa, *CASES[1])
    torch.cuda.synchronize()
    assert device_error() == 0
