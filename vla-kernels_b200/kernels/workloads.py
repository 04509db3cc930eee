"""Seeded synthetic inputs for the benchmark configurations (C1-C5).

The reference publishes no datasets for this path; its benchmarks draw seeded
torch.randn inputs (bench/bench_kernel.py:53-55, tests/*). These generators
give the shapes and value distributions of the five configurations, one
generator per tensor in the order q, k, v, and the algorithmic work counts
used for the roofline (bytes for softmax, mask-visible FLOPs for attention).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM = 64


def _gen(device, seed: int) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


# ---- softmax ---------------------------------------------------------------

def softmax_c1(device="cuda", rows: int = 4096, cols: int = 1024, seed: int = 0) -> torch.Tensor:
    """C1: fp32 [4096, 1024] ~ N(0, 3^2); exactly floor(0.05 * cols) entries of
    every row set to -inf at seeded positions; no row fully masked."""
    g = _gen(device, seed)
    x = torch.randn(rows, cols, device=device, generator=g) * 3.0
    n_inf = int(0.05 * cols)
    if n_inf:
        keys = torch.rand(rows, cols, device=device, generator=g)
        idx = keys.argsort(dim=1)[:, :n_inf]
        x.scatter_(1, idx, float("-inf"))
    return x


def softmax_c2(rows: int, cols: int, device="cuda", seed: int = 0,
               dtype=torch.bfloat16) -> torch.Tensor:
    """C2: bf16 logits ~ N(0, 4^2)."""
    g = _gen(device, seed)
    return (torch.randn(rows, cols, device=device, generator=g) * 4.0).to(dtype)


C2_ROWS = (256, 1024, 8192)
C2_COLS = (241, 1024, 4096, 16384, 32768)
C2_NARROW = (983040, 291)


def softmax_bytes(rows: int, cols: int, elem_size: int) -> int:
    """Algorithmic bytes of one softmax: one read + one write of the tensor."""
    return 2 * rows * cols * elem_size


# ---- attention -------------------------------------------------------------

@dataclass(frozen=True)
class AttnShape:
    B: int
    M: int
    N: int
    H: int
    Hkv: int
    P: int
    ds: int = 0
    de: int = 0


# C3: SmolVLA action-expert self-attention (50 action queries, 241 prefix + 50
# action keys), staircase mask; BASELINE C3 / C5
def expert_shape(B: int, N: int = 291, ds: int = 0, de: int = 0) -> AttnShape:
    return AttnShape(B=B, M=50, N=N, H=15, Hkv=5, P=241, ds=ds, de=de)


def attn_inputs(s: AttnShape, device="cuda", seed: int = 0):
    """q (B, M, H, 64), k/v (B, N, Hkv, 64) bf16 ~ N(0, 1); seeds seed, +1, +2."""
    q = torch.randn(s.B, s.M, s.H, HEAD_DIM, device=device, generator=_gen(device, seed))
    k = torch.randn(s.B, s.N, s.Hkv, HEAD_DIM, device=device, generator=_gen(device, seed + 1))
    v = torch.randn(s.B, s.N, s.Hkv, HEAD_DIM, device=device, generator=_gen(device, seed + 2))
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


def visible_pairs(M: int, N: int, P: int, ds: int = 0, de: int = 0) -> int:
    """Number of mask-visible (query row, key) pairs of one head."""
    total = 0
    for r in range(M):
        e2 = max(P, min(N, N - M + r + 1))
        total += min(ds, N) + max(0, e2 - de)
    return total


def attn_flops(s: AttnShape) -> int:
    """Algorithmic FLOPs: 2*D for QK^T plus 2*D for PV per visible pair."""
    return 4 * HEAD_DIM * s.H * s.B * visible_pairs(s.M, s.N, s.P, s.ds, s.de)


def attn_bytes(s: AttnShape) -> int:
    """Algorithmic HBM bytes: read q, k, v once and write o once (bf16)."""
    return 2 * HEAD_DIM * s.B * (2 * s.M * s.H + 2 * s.N * s.Hkv)


# C4: SmolVLA VLM-prefix attention, bidirectional over per-sample lengths
# L_b ~ U{150..241} (seeded); the compacted variant is M = N = 197, all visible.
def prefix_shape(B: int, seq: int = 241) -> AttnShape:
    return AttnShape(B=B, M=seq, N=seq, H=15, Hkv=5, P=seq)


def c4_lengths(B: int, device="cuda", seed: int = 0, lo: int = 150, hi: int = 241) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (B,), generator=g).to(device)


def varlen_flops(lengths, H: int = 15) -> int:
    """Algorithmic FLOPs of per-sample-length attention: L_b^2 visible pairs
    per (b, h)."""
    L = torch.as_tensor(lengths).to(torch.int64).cpu()
    return int(4 * HEAD_DIM * H * (L * L).sum().item())


# SigLIP vision attention site: (1, 12, 1024, 64) bf16, unmasked (B, H, M, 64)
def siglip_inputs(B: int = 1, H: int = 12, M: int = 1024, device="cuda", seed: int = 0):
    g = _gen(device, seed)
    mk = lambda: torch.randn(B, H, M, HEAD_DIM, device=device, generator=g).to(torch.bfloat16)  # noqa: E731
    return mk(), mk(), mk()
