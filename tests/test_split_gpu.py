"""GPU parity of the key-split entry points (vlak_attn_gqa_*_ws).

Small batches fill few CTAs, so the library splits each query block's keys
across CTAs and merges the partials in a second kernel. The merged output
must match the float64 oracle at the kernel's bf16 tolerance (atol 1e-2,
rtol 1.6e-2), stay within bf16 rounding of the unsplit entry points (each
split holds O / l in bf16 before the merge: atol 1e-2, rtol 1e-2 between the
two), keep rows with no visible key at exact zeros, and fall back to the
unsplit kernel, bit for bit, when the workspace is missing or too small.
"""
import numpy as np
import pytest
import torch

from oracle import gqa_attention, gqa_attention_varlen, masked_attention
from tests import capi
from tests.test_attention_gpu import check, device_error, rand

pytestmark = pytest.mark.gpu

# (B, M, N, H, Hkv, P, ds, de): the C3 / C4 sites at small batch, a dead band,
# a ragged last chunk, GQA ratios 1 / 3 / 8 and a one-chunk problem
CASES = [
    (1, 50, 291, 15, 5, 241, 0, 0),
    (8, 50, 291, 15, 5, 241, 0, 0),
    (1, 50, 291, 15, 5, 241, 196, 240),
    (1, 241, 241, 15, 5, 241, 0, 0),
    (2, 100, 700, 8, 1, 600, 100, 300),
    (1, 64, 1024, 12, 12, 1024, 0, 0),
    (1, 20, 130, 4, 4, 130, 0, 0),
    (1, 10, 60, 2, 1, 60, 0, 0),
]


def inputs(B, M, N, H, Hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return rand(B, M, H, 64, gen=g), rand(B, N, Hkv, 64, gen=g), rand(B, N, Hkv, 64, gen=g)


def close_to_unsplit(o_ws, o_plain):
    torch.testing.assert_close(o_ws.float(), o_plain.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("case", CASES)
def test_split_matches_oracle_and_unsplit(case):
    B, M, N, H, Hkv, P, ds, de = case
    q, k, v = inputs(B, M, N, H, Hkv, 3)
    st, o_ws = capi.attn_gqa_ws(q, k, v, prefix_len=P, dead_start=ds, dead_end=de)
    assert st == capi.VLAK_OK, capi.last_error()
    st, o_plain = capi.attn_gqa_plain(q, k, v, prefix_len=P, dead_start=ds, dead_end=de)
    assert st == capi.VLAK_OK, capi.last_error()
    ref = torch.from_numpy(gqa_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                         v.float().cpu().numpy(), P, ds, de))
    check(o_ws, ref)
    close_to_unsplit(o_ws, o_plain)


def test_workspace_size_follows_occupancy():
    g = torch.Generator(device="cuda").manual_seed(1)
    small = [rand(1, 50, 15, 64, gen=g), rand(1, 291, 5, 64, gen=g), rand(1, 291, 5, 64, gen=g)]
    big = [rand(64, 50, 15, 64, gen=g), rand(64, 291, 5, 64, gen=g), rand(64, 291, 5, 64, gen=g)]
    n_small = capi.workspace_size(*small, prefix_len=241)
    # C3 at B = 1: 5 query blocks, 5 chunks -> 5 splits of one chunk each
    assert n_small >= 5 * 1 * 50 * 15 * (128 + 8)
    assert capi.workspace_size(*big, prefix_len=241) == 0  # 320 blocks fill the GPU unsplit


def splits_of(case):
    """Number of key splits the library plans for a CASES entry (from the
    workspace size: 128 bytes of partial O and 8 of (m, l) per row and split)."""
    B, M, N, H, Hkv, P, ds, de = case
    q, k, v = inputs(B, M, N, H, Hkv, 0)
    return round(capi.workspace_size(q, k, v, prefix_len=P, dead_start=ds, dead_end=de) / (B * M * H * 136))


def test_cases_reach_both_merge_forms():
    # combine_splits loads up to 8 splits in one batch and loops over batches
    # of 8 beyond that: CASES holds both kinds
    counts = [splits_of(c) for c in CASES]
    assert any(2 <= n <= 8 for n in counts), counts
    assert any(n > 8 for n in counts), counts
    assert splits_of(CASES[0]) == 5  # C3 at B = 1: 5 chunks, one per split


def test_missing_or_small_workspace_runs_unsplit():
    q, k, v = inputs(1, 50, 291, 15, 5, 5)
    st, o_plain = capi.attn_gqa_plain(q, k, v, prefix_len=241)
    assert st == capi.VLAK_OK
    tiny = torch.empty(256, device="cuda", dtype=torch.uint8)
    st, o_small = capi.attn_gqa_ws(q, k, v, prefix_len=241, workspace=tiny)
    assert st == capi.VLAK_OK, capi.last_error()
    torch.cuda.synchronize()
    assert torch.equal(o_small, o_plain)


def test_misaligned_workspace_is_rejected():
    q, k, v = inputs(1, 50, 291, 15, 5, 6)
    n = capi.workspace_size(q, k, v, prefix_len=241)
    buf = torch.empty(n + 512, device="cuda", dtype=torch.uint8)
    st, _ = capi.attn_gqa_ws(q, k, v, prefix_len=241, workspace=buf[16:])
    assert st == capi.VLAK_ERR_ALIGNMENT


def test_repeated_calls_reuse_the_workspace():
    q, k, v = inputs(2, 50, 291, 15, 5, 7)
    n = capi.workspace_size(q, k, v, prefix_len=241)
    ws = torch.full((n,), 0xFF, device="cuda", dtype=torch.uint8)  # NaN bit patterns
    st, o1 = capi.attn_gqa_ws(q, k, v, prefix_len=241, workspace=ws)
    assert st == capi.VLAK_OK
    st, o2 = capi.attn_gqa_ws(q, k, v, prefix_len=241, workspace=ws)
    assert st == capi.VLAK_OK
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.isfinite(o1.float()).all()


@pytest.mark.parametrize("lengths", [(150, 241, 0), (1, 64, 65), (241, 200, 129)])
def test_varlen_split(lengths):
    # lengths ending inside, at and past chunk boundaries, and 0: later splits
    # of a short sample see no visible key and must drop out of the merge
    B = len(lengths)
    q, k, v = inputs(B, 241, 241, 15, 5, 8)
    L = torch.tensor(lengths, device="cuda", dtype=torch.int32)
    st, o_ws = capi.attn_gqa_ws(q, k, v, lengths=L)
    assert st == capi.VLAK_OK, capi.last_error()
    st, o_plain = capi.attn_gqa_plain(q, k, v, lengths=L)
    assert st == capi.VLAK_OK
    ref = torch.from_numpy(gqa_attention_varlen(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                v.float().cpu().numpy(), np.array(lengths)))
    check(o_ws, ref)
    close_to_unsplit(o_ws, o_plain)


def test_masked_split_with_rows_visible_in_one_split_only():
    B, M, N, H, Hkv = 1, 50, 291, 15, 5
    q, k, v = inputs(B, M, N, H, Hkv, 9)
    g = torch.Generator(device="cuda").manual_seed(10)
    mask = torch.rand(B, M, N, device="cuda", generator=g) < 0.3
    mask[0, :5] = False            # fully masked rows -> zeros
    mask[0, 5:10] = False
    mask[0, 5:10, 200:210] = True  # visible only inside one 64-key chunk
    mask[0, 10, 290] = True        # the last key alone
    mask[0, 10, :290] = False
    st, o_ws = capi.attn_gqa_ws(q, k, v, mask=mask)
    assert st == capi.VLAK_OK, capi.last_error()
    st, o_plain = capi.attn_gqa_plain(q, k, v, mask=mask)
    assert st == capi.VLAK_OK
    ref = torch.from_numpy(masked_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                            v.float().cpu().numpy(), mask.cpu().numpy()))
    check(o_ws, ref)
    assert (o_ws[0, :5] == 0).all()
    close_to_unsplit(o_ws, o_plain)


def test_torch_ops_take_the_split_path_at_small_batch():
    from kernels.attention import fused_attention_gqa
    q, k, v = inputs(1, 50, 291, 15, 5, 11)
    out = fused_attention_gqa(q, k, v, prefix_len=241)
    st, o_ws = capi.attn_gqa_ws(q, k, v, prefix_len=241)
    assert st == capi.VLAK_OK
    torch.cuda.synchronize()
    assert torch.equal(out, o_ws)
    assert device_error() == 0
