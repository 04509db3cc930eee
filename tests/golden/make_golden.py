"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs where a checkout of djkim9031-research/vla-kernels is available: it
imports the reference's own oracle functions from that checkout and reads its
real-mask fixture. The checkout's root comes from --reference, else from the
environment variable VLAK_REFERENCE; there is no default. The outputs are
small .npz files committed beside this script; the tests read only those.

  python tests/golden/make_golden.py --reference PATH
  VLAK_REFERENCE=PATH python tests/golden/make_golden.py

Inputs are regenerated from recorded seeds with torch's CPU generator; a
SHA-256 of the input bytes is stored so a generator change is detected.

Fixtures:
  softmax_golden.npz   torch.softmax outputs (the oracle of
                       tests/test_softmax.py:24-30), incl. -inf entries and
                       the extreme-values case of :55-61
  attention_golden.npz ref_attn outputs (tests/test_attention_gqa.py:12-25)
                       for a grid of (B, M, N, H, Hkv, P, ds, de) cases from
                       its CASES (:43-54), scaled to small sizes, plus one case
                       with fully masked rows (NaN in ref_attn)
  masks_golden.npz     the three masks of results/real_masks.pt (packed bits)
                       and what _analytic_params (vla/variants.py:236-255)
                       solves them to
  sdpa_golden.npz      ref_sdpa outputs (tests/test_attention.py:25-30) for the
                       (B, H, M, 64) op: the SmolVLA prefix/causal pattern of
                       smolvla_mask (:33-40), the real 241x241 prefix mask
                       (pad rows and a block-causal state token), a random mask
                       and no mask; fully masked rows are NaN there
  varlen_golden.npz    ref_sdpa outputs for per-sample lengths (the C4 prefix
                       site), GQA by repeating kv heads as ref_attn does
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (B, M, N, H, Hkv, P, ds, de, seed)
ATTN_CASES = [
    (1, 50, 241, 15, 5, 241, 196, 240, 0),   # expert cross site, real mask
    (1, 50, 291, 15, 5, 241, 196, 240, 1),   # expert self site, real mask
    (1, 33, 65, 4, 2, 40, 8, 16, 2),         # one past tile boundaries
    (2, 37, 127, 8, 8, 100, 20, 44, 3),      # MHA (G=1), odd sizes
    (1, 32, 64, 4, 2, 64, 0, 0, 4),          # exact tile boundaries
    (1, 40, 128, 6, 2, 128, 32, 64, 5),      # dead band covers 2 fragments
    (1, 12, 16, 2, 1, 12, 0, 12, 6),         # rows 0-7 see no key
]


# (B, H, M, N, mask kind, seed) for the (B, H, M, 64) op
SDPA_CASES = [
    (1, 3, 50, 291, "smolvla241", 10),
    (2, 2, 33, 65, "smolvla32", 11),
    (1, 2, 241, 241, "real_prefix", 12),
    (2, 2, 17, 33, "random", 13),
    (1, 2, 40, 70, "none", 14),
]
# (B, M, N, H, Hkv, lengths, seed) for per-sample lengths
VARLEN_CASES = [
    (2, 241, 241, 3, 1, (150, 241), 20),
    (2, 40, 40, 3, 1, (0, 17), 21),
]


def smolvla_pattern(M, N, prefix):
    """The prefix-bidirectional + causal-suffix pattern of smolvla_mask
    (tests/test_attention.py:33-40), built on the CPU."""
    m = torch.zeros(M, N, dtype=torch.bool)
    m[:, :prefix] = True
    start = N - M
    for i in range(M):
        m[i, prefix:start + i + 1] = True
    return m


def sdpa_mask(kind, B, M, N, seed, real_masks):
    if kind == "none":
        return None
    if kind.startswith("smolvla"):
        return smolvla_pattern(M, N, int(kind[len("smolvla"):]))[None].expand(B, M, N).contiguous()
    if kind == "real_prefix":
        return real_masks[(M, N)][None].expand(B, M, N).contiguous()
    g = torch.Generator().manual_seed(seed + 1000)
    m = torch.rand(B, M, N, generator=g) < 0.6
    m[0, 3] = False  # one row sees no key
    return m


def bhmd_inputs(B, H, M, N, seed):
    """Seeded bf16-valued q/k/v in (B, H, seq, 64), held as fp32."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, M, 64, generator=g).to(torch.bfloat16).float()
    k = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).float()
    v = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).float()
    return q, k, v


def attn_inputs(B, M, N, H, Hkv, seed):
    """Seeded bf16 q/k/v in the op's natural layouts (N(0,1), one stream)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, M, H, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, Hkv, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, Hkv, 64, generator=g).to(torch.bfloat16)
    return q, k, v


def softmax_inputs():
    cases = {}
    for i, (r, c) in enumerate([(1, 16), (8, 31), (128, 64), (16, 1000), (4, 4096)]):
        g = torch.Generator().manual_seed(100 + i)
        cases[f"randn_{r}x{c}"] = torch.randn(r, c, generator=g)
    # C1-style rows: N(0, 3^2) with 51 of 1024 entries per row at -inf
    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 1024, generator=g) * 3.0
    for row in range(16):
        idx = torch.randperm(1024, generator=g)[:51]
        x[row, idx] = float("-inf")
    cases["c1_16x1024_neginf"] = x
    cases["extreme"] = torch.tensor([[1000.0, 1001.0, 999.0, -1000.0]])
    return cases


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VLAK_REFERENCE"),
                    help="root of a djkim9031-research/vla-kernels checkout "
                         "(default: $VLAK_REFERENCE)")
    a = ap.parse_args()
    if not a.reference or not os.path.isfile(os.path.join(a.reference, "tests", "test_attention_gqa.py")):
        ap.error("give the reference checkout with --reference PATH or VLAK_REFERENCE=PATH "
                 f"(got {a.reference!r}, which holds no tests/test_attention_gqa.py)")
    sys.path.insert(0, a.reference)
    from tests.test_attention_gqa import ref_attn  # reference oracle
    from vla.variants import _analytic_params      # reference mask solver
    from tests.test_attention import ref_sdpa       # reference SDPA oracle

    # ---- softmax
    out = {}
    for name, x in softmax_inputs().items():
        out[f"{name}__sha256"] = np.array(digest(x))
        out[f"{name}__y"] = torch.softmax(x.float(), dim=-1).numpy()
    np.savez_compressed(os.path.join(HERE, "softmax_golden.npz"), **out)

    # ---- attention
    out = {"cases": np.array(ATTN_CASES, dtype=np.int64)}
    for i, (B, M, N, H, Hkv, P, ds, de, seed) in enumerate(ATTN_CASES):
        q, k, v = attn_inputs(B, M, N, H, Hkv, seed)
        ref = ref_attn(q, k, v, P, ds, de)
        out[f"c{i}__out"] = ref.float().numpy()
        out[f"c{i}__sha256"] = np.array(digest(q, k, v))
    np.savez_compressed(os.path.join(HERE, "attention_golden.npz"), **out)

    # ---- real masks
    masks = torch.load(os.path.join(a.reference, "results", "real_masks.pt"), weights_only=True)
    out = {}
    for m in masks.values():
        M, N = m.shape
        key = f"m{M}x{N}"
        out[f"{key}__bits"] = np.packbits(m.numpy().astype(np.uint8).ravel())
        out[f"{key}__shape"] = np.array([M, N])
        par = _analytic_params(m.cpu(), M, N)
        out[f"{key}__params"] = np.array(par if par is not None else (-1, -1, -1))
    np.savez_compressed(os.path.join(HERE, "masks_golden.npz"), **out)

    # ---- (B, H, M, 64) op with bool / pattern / no masks
    real = {tuple(m.shape): m.cpu().bool() for m in masks.values()}
    out = {}
    for i, (B, H, M, N, kind, seed) in enumerate(SDPA_CASES):
        q, k, v = bhmd_inputs(B, H, M, N, seed)
        mask = sdpa_mask(kind, B, M, N, seed, real)
        out[f"s{i}__out"] = ref_sdpa(q, k, v, mask).numpy()
        out[f"s{i}__sha256"] = np.array(digest(q, k, v))
        if mask is not None:
            out[f"s{i}__mask"] = np.packbits(mask.numpy().astype(np.uint8).ravel())
    np.savez_compressed(os.path.join(HERE, "sdpa_golden.npz"), **out)

    # ---- per-sample lengths (GQA, natural layouts)
    out = {}
    for i, (B, M, N, H, Hkv, lengths, seed) in enumerate(VARLEN_CASES):
        q, k, v = attn_inputs(B, M, N, H, Hkv, seed)
        L = torch.tensor(lengths)[:, None, None]
        vis = (torch.arange(N)[None, None, :] < L) & (torch.arange(M)[None, :, None] < L)
        G = H // Hkv
        qh = q.float().transpose(1, 2)
        kh = k.float().transpose(1, 2).repeat_interleave(G, dim=1)
        vh = v.float().transpose(1, 2).repeat_interleave(G, dim=1)
        out[f"v{i}__out"] = ref_sdpa(qh, kh, vh, vis).transpose(1, 2).numpy()
        out[f"v{i}__sha256"] = np.array(digest(q, k, v))
    np.savez_compressed(os.path.join(HERE, "varlen_golden.npz"), **out)
    for f in ("softmax_golden.npz", "attention_golden.npz", "masks_golden.npz", "sdpa_golden.npz",
              "varlen_golden.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
