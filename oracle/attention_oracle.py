"""GQA attention oracle with the analytic SmolVLA mask (test infrastructure only).

Restates:
  * the mask predicate of the v3/v4 kernels and of their oracle
    (kernels/attention/fused_attention.cu:378-398, :437-445;
    tests/test_attention_gqa.py:20-23):
        visible(r, c) = c < P ? (c < ds or c >= de) : c <= (N - M) + r
  * ref_attn (tests/test_attention_gqa.py:12-25): GQA by repeating each kv
    head over its G query heads, scores scaled by D**-0.5 (or the given
    scale), masked softmax, times V -- here in float64;
  * _analytic_params (vla/variants.py:236-255): solve a captured (M, N) bool
    mask for (P, ds, de), requiring exact equality;
  * ref_sdpa (tests/test_attention.py:25-30) and the masking rules of the
    (B, H, M, 64) op vlak::fused_attention (fused_attention.cu:525-598);
  * the per-sample-length mask of the prefix site (C4), which the reference
    hands to SDPA as a materialised mask.
Rows with no visible key are exact zeros (the contract of the B200 build;
the reference's torch oracle yields NaN for them).
"""
from __future__ import annotations

import numpy as np


def analytic_visible(M: int, N: int, P: int, ds: int, de: int) -> np.ndarray:
    """(M, N) bool mask of the analytic two-boundary predicate."""
    r = np.arange(M)[:, None]
    c = np.arange(N)[None, :]
    return np.where(c < P, (c < ds) | (c >= de), c <= (N - M) + r)


def varlen_visible(lengths, M: int, N: int) -> np.ndarray:
    """(B, M, N) bool mask of per-sample lengths: c < L_b and r < L_b, with
    L_b clamped to [0, N] (the C4 prefix site; the reference builds this
    mask for SDPA, docs/attention.md:276-278)."""
    L = np.clip(np.asarray(lengths, dtype=np.int64), 0, N)[:, None, None]
    r = np.arange(M)[None, :, None]
    c = np.arange(N)[None, None, :]
    return (c < L) & (r < L)


def masked_attention(q, k, v, vis, scale: float | None = None) -> np.ndarray:
    """q (B, M, H, D), k/v (B, N, Hkv, D), vis (B, M, N) or (M, N) bool
    (True = attend) -> (B, M, H, D) float64. Query head h reads kv head
    h // (H / Hkv); scores scaled by D**-0.5 unless a positive scale is given
    (ref_attn, tests/test_attention_gqa.py:12-25; ref_sdpa,
    tests/test_attention.py:25-30). Rows with no visible key are zeros."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, M, H, D = q.shape
    N, Hkv = k.shape[1], k.shape[2]
    if H % Hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    G = H // Hkv
    sc = D ** -0.5 if scale is None or scale <= 0 else scale
    if N == 0 or M == 0 or B == 0:
        return np.zeros((B, M, H, D))
    vis = np.asarray(vis, dtype=bool)
    vis = (vis[None] if vis.ndim == 2 else vis)[:, None]          # (B|1, 1, M, N)
    qh = q.transpose(0, 2, 1, 3)                                   # (B, H, M, D)
    kh = np.repeat(k.transpose(0, 2, 1, 3), G, axis=1)             # (B, H, N, D)
    vh = np.repeat(v.transpose(0, 2, 1, 3), G, axis=1)
    s = np.matmul(qh, kh.transpose(0, 1, 3, 2)) * sc               # (B, H, M, N)
    s = np.where(vis, s, -np.inf)
    mx = s.max(axis=-1, keepdims=True)
    any_vis = np.isfinite(mx)
    with np.errstate(invalid="ignore"):
        e = np.where(vis, np.exp(s - np.where(any_vis, mx, 0.0)), 0.0)
    l = e.sum(axis=-1, keepdims=True)
    p = np.where(l > 0, e / np.where(l > 0, l, 1.0), 0.0)
    return np.matmul(p, vh).transpose(0, 2, 1, 3)                  # (B, M, H, D)


def gqa_attention(q, k, v, prefix_len: int | None = None, dead_start: int = 0,
                  dead_end: int = 0, scale: float | None = None) -> np.ndarray:
    """q (B, M, H, D), k/v (B, N, Hkv, D) -> (B, M, H, D) float64 under the
    analytic mask."""
    M, N = np.shape(q)[1], np.shape(k)[1]
    P = N if prefix_len is None or prefix_len < 0 else prefix_len
    return masked_attention(q, k, v, analytic_visible(M, N, P, dead_start, dead_end), scale)


def gqa_attention_varlen(q, k, v, lengths, scale: float | None = None) -> np.ndarray:
    """Per-sample-length GQA attention (vlak::fused_attention_gqa_varlen)."""
    return masked_attention(q, k, v, varlen_visible(lengths, np.shape(q)[1], np.shape(k)[1]),
                            scale)


def sdpa_bhmd(q, k, v, attn_mask=None, prefix_len: int | None = None,
              scale: float | None = None) -> np.ndarray:
    """vlak::fused_attention semantics on (B, H, M, D) tensors
    (kernels/attention/fused_attention.cu:525-598): prefix_len >= 0 selects the
    analytic mask c < P or c <= (N - M) + r (fused_attention.cu:166-232) and
    wins over attn_mask; else attn_mask (B, M, N) bool; else unmasked."""
    q = np.asarray(q, dtype=np.float64).transpose(0, 2, 1, 3)
    k = np.asarray(k, dtype=np.float64).transpose(0, 2, 1, 3)
    v = np.asarray(v, dtype=np.float64).transpose(0, 2, 1, 3)
    M, N = q.shape[1], k.shape[1]
    if prefix_len is not None and prefix_len >= 0:
        vis = analytic_visible(M, N, min(prefix_len, N), 0, 0)
    elif attn_mask is not None:
        vis = np.asarray(attn_mask, dtype=bool)
    else:
        vis = np.ones((M, N), dtype=bool)
    return masked_attention(q, k, v, vis, scale).transpose(0, 2, 1, 3)


def gqa_attention_torch_cpu(q, k, v, prefix_len: int | None = None, dead_start: int = 0,
                            dead_end: int = 0, scale: float | None = None):
    """The reference's CPU path, for timing on host cores: torch SDPA with a
    bool mask and GQA by repeat_interleave (BASELINE plan), fp32 math."""
    import torch
    import torch.nn.functional as F

    B, M, H, D = q.shape
    N, Hkv = k.shape[1], k.shape[2]
    G = H // Hkv
    P = N if prefix_len is None or prefix_len < 0 else prefix_len
    sc = D ** -0.5 if scale is None or scale <= 0 else scale
    r = torch.arange(M)[:, None]
    c = torch.arange(N)[None, :]
    vis = torch.where(c < P, (c < dead_start) | (c >= dead_end), c <= (N - M) + r)
    qf = q.float().permute(0, 2, 1, 3)
    kf = k.float().permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    vf = v.float().permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    o = F.scaled_dot_product_attention(qf, kf, vf, attn_mask=vis, scale=sc)
    return o.permute(0, 2, 1, 3)


def solve_analytic_params(mask: np.ndarray):
    """(P, ds, de) whose analytic predicate equals ``mask`` exactly, else None.

    Candidates P = N (no suffix) then P = N - M (a suffix of M rows); the dead
    band is the span of prefix columns no row can see.
    """
    m2 = np.asarray(mask, dtype=bool)
    M, N = m2.shape
    for P in dict.fromkeys([N, N - M]):
        if P <= 0:
            continue
        pre = m2[:, :P]
        dead = np.flatnonzero(~pre.any(axis=0))
        ds, de = (int(dead.min()), int(dead.max()) + 1) if dead.size else (0, 0)
        if np.array_equal(analytic_visible(M, N, P, ds, de), m2):
            return (P, ds, de)
    return None
