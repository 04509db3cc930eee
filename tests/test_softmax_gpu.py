"""GPU parity of vlak::softmax against the CPU oracle (and torch.softmax).

Tolerances: fp32 max relative error <= 1e-6; fp16/bf16 atol 1e-2, rtol 1.6e-2
against the fp32 oracle. Versions 0-4 all run the same
checks, through the torch op and through the C ABI.
"""
import numpy as np
import pytest
import torch

from kernels import workloads as wl
from kernels.softmax import VERSIONS, softmax
from oracle import softmax_rows
from tests import capi

pytestmark = pytest.mark.gpu

SHAPES = [(1, 16), (8, 31), (128, 64), (1024, 128), (256, 1000), (4, 4096),
          (33, 241), (7, 291), (5, 2049), (3, 8193), (2, 32768), (1, 40000), (64, 1)]
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def check(out, x, dtype):
    ref = softmax_rows(x.float().cpu().numpy())
    got = out.double().cpu().numpy()
    if dtype in (torch.float32, torch.float64):
        pos = ref > 0
        rel = np.abs(got[pos] - ref[pos]) / ref[pos]
        assert rel.max(initial=0) <= 1e-6, f"max rel err {rel.max()}"
        assert np.array_equal(got[~pos], ref[~pos])
    else:
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(ref),
                                   atol=1e-2, rtol=1.6e-2)


@pytest.mark.parametrize("version", list(VERSIONS))
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_matches_oracle(version, dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(*shape, device="cuda", generator=g) * 3).to(dtype)
    check(softmax(x, version=version), x, dtype)


@pytest.mark.parametrize("version", [0, 1, 2, 3, 4, 7])
def test_c1_full_size_fp32_with_neg_inf(version):
    x = wl.softmax_c1()
    assert torch.isinf(x).sum(1).eq(51).all()
    out = softmax(x, version)
    check(out, x, torch.float32)
    assert (out[torch.isinf(x)] == 0).all()


@pytest.mark.parametrize("version", list(VERSIONS))
def test_c1_matches_torch_softmax_fp32(version):
    x = wl.softmax_c1()
    ref = torch.softmax(x, -1)
    out = softmax(x, version)
    pos = ref > 0
    rel = ((out[pos].double() - ref[pos].double()).abs() / ref[pos].double()).max().item()
    assert rel <= 1e-6


@pytest.mark.parametrize("rows", wl.C2_ROWS)
@pytest.mark.parametrize("cols", wl.C2_COLS)
def test_c2_sweep_bf16(rows, cols):
    x = wl.softmax_c2(rows, cols)
    out = softmax(x, "auto")
    # full check on a subset of rows (oracle cost), row sums everywhere
    idx = torch.arange(0, rows, max(1, rows // 64), device="cuda")
    check(out[idx], x[idx], torch.bfloat16)
    sums = out.float().sum(-1)
    assert ((sums - 1).abs() < 2e-2 + cols * 4e-3 * 2 ** -8).all()


# More wide rows than the GPU holds blocks for at once (several waves of one
# block per row): sampled rows against the oracle, every row's sum, and rows
# of whole 16-byte vectors exactly as a short call of the same rows computes
# them (a ragged row's segmentation depends on its address, so a short call of
# such rows may take another path).
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(1024, 32768), (4097, 8192), (3000, 1032), (2000, 4096),
                                       (700, 20008), (700, 20001)])
def test_many_wide_rows_match_short_calls(rows, cols, dtype):
    g = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 4).to(dtype)
    out = softmax(x, 4)
    idx = torch.cat([torch.arange(0, 8), torch.arange(rows - 8, rows),
                     torch.randint(0, rows, (48,), generator=torch.Generator().manual_seed(2))])
    check(out[idx.cuda()], x[idx.cuda()], dtype)
    sums = out.float().sum(-1)
    assert ((sums - 1).abs() < 2e-2 + cols * 4e-3 * 2 ** -8).all()
    if cols % 8 == 0:
        for r0 in (0, rows // 2, rows - 16):
            assert torch.equal(out[r0:r0 + 16], softmax(x[r0:r0 + 16], 4)), r0


def test_c2_narrow_many_rows_bf16():
    rows, cols = wl.C2_NARROW
    x = wl.softmax_c2(rows, cols, seed=3)
    out = softmax(x, "auto")
    idx = torch.randint(0, rows, (2048,), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    check(out[idx], x[idx], torch.bfloat16)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("version", list(VERSIONS))
def test_extreme_values_are_stable(version):
    # tests/test_softmax.py:55-61
    x = torch.tensor([[1000.0, 1001.0, 999.0, -1000.0]], device="cuda")
    out = softmax(x, version=version)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.sum(dim=-1), torch.ones(1, device="cuda"), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("version", list(VERSIONS))
def test_all_neg_inf_row_is_nan_like_torch(version):
    x = torch.randn(3, 300, device="cuda")
    x[1] = float("-inf")
    out = softmax(x, version)
    assert torch.isnan(out[1]).all() and torch.isfinite(out[[0, 2]]).all()


@pytest.mark.parametrize("version", list(VERSIONS))
@pytest.mark.parametrize("dtype", DTYPES)
def test_offset_view_input(version, dtype):
    # x starts 1 element past a 16-byte boundary while y is aligned
    base = torch.randn(37 * 291 + 1, device="cuda").to(dtype)
    x = base[1:].view(37, 291)
    check(softmax(x, version), x, dtype)


def test_float64_input_computed_like_reference():
    x = torch.randn(16, 777, device="cuda", dtype=torch.float64)
    out = softmax(x, 4)
    assert out.dtype == torch.float64
    check(out.float(), x.float(), torch.float32)


def test_empty_tensors():
    for shape in [(0, 16), (16, 0)]:
        x = torch.empty(*shape, device="cuda")
        assert softmax(x, 4).shape == shape


def test_non_contiguous_input_is_made_contiguous():
    x = torch.randn(64, 300, device="cuda").t()
    out = softmax(x, 1)
    assert out.is_contiguous()
    check(out, x.contiguous(), torch.float32)


@pytest.mark.parametrize("version", list(VERSIONS))
@pytest.mark.parametrize("dtype", DTYPES)
def test_through_c_abi(version, dtype):
    x = (torch.randn(100, 1000, device="cuda") * 4).to(dtype)
    st, y = capi.softmax(x, VERSIONS[version])
    assert st == capi.VLAK_OK, capi.last_error()
    torch.cuda.synchronize()
    check(y, x, dtype)
    assert torch.equal(y, softmax(x, version))


def test_registered_op_and_compile():
    # tests/test_softmax.py:64-90
    x = torch.randn(16, 128, device="cuda")
    torch.testing.assert_close(torch.ops.vlak.softmax(x, 1), torch.softmax(x, -1),
                               rtol=1e-5, atol=1e-6)

    def f(x):
        return softmax(x, "v4") * 2.0

    softmax(x, "v4")
    out = torch.compile(f, fullgraph=True)(x)
    torch.testing.assert_close(out, torch.softmax(x, -1) * 2.0, rtol=1e-4, atol=1e-5)


def test_patch_kernels_style_call():
    # vla/patch_kernels.py:26-36 reshapes N-d last-dim softmax to 2D and calls "auto"
    x = torch.randn(2, 15, 50, 291, device="cuda")
    out = softmax(x.reshape(-1, 291), "auto").reshape(x.shape)
    torch.testing.assert_close(out, torch.softmax(x, -1), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("version", list(VERSIONS))
@pytest.mark.parametrize("shape", [(64, 291), (8, 1024), (8, 4096), (4, 16384), (2, 32768)])
def test_bf16_keeps_tail_probabilities(version, shape):
    """A wide logit spread puts most probabilities far below 2^-24. Each must
    come out within a relative tolerance of the fp64 oracle, as torch.softmax
    keeps them, not flushed to zero. Bound: the exp and the normalised value
    are each rounded to bf16 once (2 x 2^-9), plus fp32 arithmetic: 1e-2."""
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.rand(*shape, device="cuda", generator=g) * -60.0).to(torch.bfloat16)
    out = softmax(x, version=version).double().cpu().numpy()
    ref = softmax_rows(x.float().cpu().numpy())
    keep = ref >= 1e-36  # bf16 normal range, away from its subnormals
    assert keep.mean() > 0.5
    rel = np.abs(out[keep] - ref[keep]) / ref[keep]
    assert rel.max() <= 1e-2, f"max rel err {rel.max()} on probabilities down to {ref[keep].min()}"
    assert (out[keep] > 0).all(), "a probability torch keeps was flushed to zero"


@pytest.mark.parametrize("which", ["cudnn", "cub"])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 16), (33, 241), (256, 1000), (4, 4096), (2, 32768)])
def test_library_comparators_match_oracle(which, dtype, shape):
    """softmax_cudnn / softmax_cub (benchmark bars) compute the same softmax:
    fp32 within torch's fp32 tolerance (rtol 1e-5, atol 1e-6), fp16 / bf16
    within atol 1e-2, rtol 1.6e-2 of the fp64 oracle."""
    from kernels.softmax import softmax_cub, softmax_cudnn

    fn = softmax_cudnn if which == "cudnn" else softmax_cub
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.randn(*shape, device="cuda", generator=g) * 3).to(dtype)
    out = fn(x).double().cpu()
    ref = torch.from_numpy(softmax_rows(x.float().cpu().numpy()))
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)
    else:
        torch.testing.assert_close(out, ref, atol=1e-2, rtol=1.6e-2)
