"""Pin the CPU oracle to the reference: its outputs must match the golden
vectors produced by the reference's own oracles (tests/golden/make_golden.py).
CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import analytic_visible, gqa_attention, softmax_rows, solve_analytic_params
from tests.golden.make_golden import ATTN_CASES, attn_inputs, digest, softmax_inputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def sm_golden():
    return np.load(os.path.join(GOLDEN, "softmax_golden.npz"))


@pytest.fixture(scope="module")
def attn_golden():
    return np.load(os.path.join(GOLDEN, "attention_golden.npz"))


@pytest.fixture(scope="module")
def mask_golden():
    return np.load(os.path.join(GOLDEN, "masks_golden.npz"))


@pytest.mark.parametrize("name", list(softmax_inputs()))
def test_softmax_oracle_matches_torch_softmax(sm_golden, name):
    x = softmax_inputs()[name]
    assert digest(x) == str(sm_golden[f"{name}__sha256"]), "input generator changed"
    y_ref = sm_golden[f"{name}__y"].astype(np.float64)
    y = softmax_rows(x.numpy())
    # torch.softmax fp32 vs the exact fp32 pipeline: a few ulp
    pos = y_ref > 0
    rel = np.abs(y[pos] - y_ref[pos]) / y_ref[pos]
    assert rel.max() <= 1e-6, rel.max()
    assert np.array_equal(y_ref == 0, y == 0)   # -inf entries are exact zeros


def test_softmax_oracle_extreme_values_sum_to_one():
    # tests/test_softmax.py:55-61
    y = softmax_rows(np.array([[1000.0, 1001.0, 999.0, -1000.0]]))
    assert np.isfinite(y).all() and abs(y.sum() - 1.0) < 1e-12


def test_softmax_oracle_all_neg_inf_row_is_nan_like_torch():
    x = np.full((1, 8), -np.inf, dtype=np.float32)
    assert np.isnan(softmax_rows(x)).all()
    assert torch.isnan(torch.softmax(torch.from_numpy(x), -1)).all()


@pytest.mark.parametrize("idx", range(len(ATTN_CASES)))
def test_attention_oracle_matches_ref_attn(attn_golden, idx):
    B, M, N, H, Hkv, P, ds, de, seed = ATTN_CASES[idx]
    q, k, v = attn_inputs(B, M, N, H, Hkv, seed)
    assert digest(q, k, v) == str(attn_golden[f"c{idx}__sha256"]), "input generator changed"
    ref = attn_golden[f"c{idx}__out"].astype(np.float64)
    out = gqa_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), P, ds, de)
    nan_rows = np.isnan(ref).all(axis=-1)
    # the reference oracle yields NaN for rows that see no key; the contract
    # of this build is exact zeros there
    assert np.array_equal(out[nan_rows], np.zeros_like(out[nan_rows]))
    assert not np.isnan(ref[~nan_rows]).any()
    np.testing.assert_allclose(out[~nan_rows], ref[~nan_rows], rtol=1e-5, atol=1e-5)


def test_golden_grid_has_fully_masked_rows(attn_golden):
    ref = attn_golden[f"c{len(ATTN_CASES) - 1}__out"]
    assert np.isnan(ref).all(axis=-1).any()


@pytest.mark.parametrize("key", ["m241x241", "m50x291", "m50x241"])
def test_real_masks_solve_like_reference(mask_golden, key):
    M, N = (int(x) for x in mask_golden[f"{key}__shape"])
    bits = np.unpackbits(mask_golden[f"{key}__bits"])[: M * N].reshape(M, N).astype(bool)
    ref_par = tuple(int(x) for x in mask_golden[f"{key}__params"])
    par = solve_analytic_params(bits)
    assert (par if par is not None else (-1, -1, -1)) == ref_par
    if par is not None:
        # the analytic predicate reproduces the real mask bit-exactly
        assert np.array_equal(analytic_visible(M, N, *par), bits)


def test_expert_masks_are_the_smolvla_params(mask_golden):
    for key in ("m50x291", "m50x241"):
        assert tuple(mask_golden[f"{key}__params"]) == (241, 196, 240)


def test_prefix_mask_has_padding_rows_and_block_causal_state(mask_golden):
    M, N = 241, 241
    m = np.unpackbits(mask_golden["m241x241__bits"])[: M * N].reshape(M, N).astype(bool)
    assert (~m[196:240]).all()                      # 44 padding query rows
    assert m[:196, :196].all() and not m[:196, 240].any()
    assert m[240, :196].all() and m[240, 240]       # state token


def test_gqa_head_mapping():
    # query head h must read kv head h // G
    rng = np.random.default_rng(0)
    B, M, N, H, Hkv = 1, 3, 5, 6, 2
    q = rng.standard_normal((B, M, H, 8))
    k = rng.standard_normal((B, N, Hkv, 8))
    v = rng.standard_normal((B, N, Hkv, 8))
    o = gqa_attention(q, k, v, scale=0.3)
    for h in range(H):
        kv = h // (H // Hkv)
        s = q[0, :, h] @ k[0, :, kv].T * 0.3
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        np.testing.assert_allclose(o[0, :, h], p @ v[0, :, kv], rtol=1e-12)


def test_zero_keys_give_zero_rows():
    q = np.ones((1, 2, 2, 64))
    k = np.ones((1, 0, 1, 64))
    assert np.array_equal(gqa_attention(q, k, k), np.zeros((1, 2, 2, 64)))


# ---- the (B, H, M, 64) op and per-sample lengths (ref_sdpa fixtures)

from oracle import gqa_attention_varlen, sdpa_bhmd  # noqa: E402
from tests.golden.make_golden import SDPA_CASES, VARLEN_CASES, bhmd_inputs  # noqa: E402


@pytest.fixture(scope="module")
def sdpa_golden():
    return np.load(os.path.join(GOLDEN, "sdpa_golden.npz"))


@pytest.fixture(scope="module")
def varlen_golden():
    return np.load(os.path.join(GOLDEN, "varlen_golden.npz"))


def golden_mask(g, i, B, M, N):
    key = f"s{i}__mask"
    if key not in g:
        return None
    return np.unpackbits(g[key])[: B * M * N].reshape(B, M, N).astype(bool)


def assert_matches_nan_as_zero(out, ref, tol=1e-5):
    nan_rows = np.isnan(ref).all(axis=-1)
    assert np.array_equal(out[nan_rows], np.zeros_like(out[nan_rows]))
    np.testing.assert_allclose(out[~nan_rows], ref[~nan_rows], rtol=tol, atol=tol)


@pytest.mark.parametrize("idx", range(len(SDPA_CASES)))
def test_sdpa_oracle_matches_ref_sdpa(sdpa_golden, idx):
    B, H, M, N, kind, seed = SDPA_CASES[idx]
    q, k, v = bhmd_inputs(B, H, M, N, seed)
    assert digest(q, k, v) == str(sdpa_golden[f"s{idx}__sha256"]), "input generator changed"
    mask = golden_mask(sdpa_golden, idx, B, M, N)
    out = sdpa_bhmd(q.numpy(), k.numpy(), v.numpy(), attn_mask=mask)
    assert_matches_nan_as_zero(out, sdpa_golden[f"s{idx}__out"].astype(np.float64))


def test_real_prefix_mask_has_pad_rows_and_block_causal_state(sdpa_golden):
    idx = [c[4] for c in SDPA_CASES].index("real_prefix")
    B, H, M, N, _, _ = SDPA_CASES[idx]
    m = golden_mask(sdpa_golden, idx, B, M, N)[0]
    assert (~m[196:240]).all()               # 44 pad rows see nothing
    assert m[240, :196].all() and m[240, 240] and not m[240, 196:240].any()
    assert solve_analytic_params(m) is None  # not expressible analytically


@pytest.mark.parametrize("idx", [i for i, c in enumerate(SDPA_CASES) if c[4].startswith("smolvla")])
def test_sdpa_oracle_analytic_prefix_equals_pattern_mask(sdpa_golden, idx):
    B, H, M, N, kind, seed = SDPA_CASES[idx]
    q, k, v = bhmd_inputs(B, H, M, N, seed)
    mask = golden_mask(sdpa_golden, idx, B, M, N)
    P = int(kind[len("smolvla"):])
    a = sdpa_bhmd(q.numpy(), k.numpy(), v.numpy(), prefix_len=P)
    b = sdpa_bhmd(q.numpy(), k.numpy(), v.numpy(), attn_mask=mask)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("idx", range(len(VARLEN_CASES)))
def test_varlen_oracle_matches_ref_sdpa(varlen_golden, idx):
    B, M, N, H, Hkv, lengths, seed = VARLEN_CASES[idx]
    q, k, v = attn_inputs(B, M, N, H, Hkv, seed)
    assert digest(q, k, v) == str(varlen_golden[f"v{idx}__sha256"]), "input generator changed"
    out = gqa_attention_varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(), lengths)
    assert_matches_nan_as_zero(out, varlen_golden[f"v{idx}__out"].astype(np.float64))
