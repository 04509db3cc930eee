"""GQA-native fused attention on B200 (sm_100a) behind ``torch.ops.vlak``.

Same API as the reference module (kernels/attention/__init__.py):
``fused_attention`` (the (B, H, M, 64) op with a bool or analytic mask),
``fused_attention_gqa`` and ``fused_attention_gqa_v4`` with their fake (meta)
implementations and register guards, so ``vla/variants.py`` routes to them
unchanged and each call traces as one node under ``torch.compile``. One
additive op has no counterpart there: ``fused_attention_gqa_varlen``
(per-sample lengths, the prefix-attention site the reference leaves on SDPA).

The bf16 ops run one tcgen05 kernel (vla-kernels_b200/csrc/attention_gqa.cu):
QK^T and PV on the 5th-generation tensor cores with accumulators in tensor
memory, Q/K/V staged by TMA, the G query heads of a kv head sharing its K/V
tiles, the online softmax in registers and the prefix / dead-band / causal
mask computed from indices.
"""
from __future__ import annotations

from functools import lru_cache

import torch

from .. import _native


@lru_cache(maxsize=1)
def _ext():
    _native.load_ops()
    # the ops return CONTIGUOUS tensors of q's shape; the fakes must promise
    # the same strides (kernels/attention/__init__.py:26-30)
    torch.library.register_fake("vlak::fused_attention")(
        lambda q, k, v, scale=-1.0, attn_mask=None, prefix_len=-1:
            torch.empty(q.shape, dtype=q.dtype, device=q.device))
    torch.library.register_fake("vlak::fused_attention_gqa")(
        lambda q, k, v, scale=-1.0, prefix_len=-1, dead_start=0, dead_end=0:
            torch.empty(q.shape, dtype=q.dtype, device=q.device))
    torch.library.register_fake("vlak::fused_attention_gqa_varlen")(
        lambda q, k, v, lengths, scale=-1.0:
            torch.empty(q.shape, dtype=q.dtype, device=q.device))
    return torch.ops.vlak


@lru_cache(maxsize=1)
def _ext_v4():
    _native.load_ops()
    torch.library.register_fake("vlak::fused_attention_gqa_v4")(
        lambda q, k, v, scale=-1.0, prefix_len=-1, dead_start=0, dead_end=0:
            torch.empty(q.shape, dtype=q.dtype, device=q.device))
    return torch.ops.vlak


_registered = False
_registered_v4 = False


def _ensure_registered():
    global _registered
    if not _registered:
        _ext()
        _registered = True


def _ensure_registered_v4():
    global _registered_v4
    if not _registered_v4:
        _ext_v4()
        _registered_v4 = True


def fused_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    scale: float | None = None,
                    attn_mask: torch.Tensor | None = None,
                    prefix_len: int | None = None) -> torch.Tensor:
    """SDPA for (B, H, M, 64) tensors (kernels/attention/__init__.py:80-101).

    Masking, in preference order:
      prefix_len=P  analytic: col visible iff col < P or col <= (N - M) + row;
                    bf16 (tensor-core) path only.
      attn_mask     generic (B, M, N) bool, broadcast over heads.
      neither       unmasked.
    bf16 runs on the tensor cores; fp32 / fp16 / fp64 on the CUDA cores with
    fp32 math. Rows with no visible key are exact zeros.
    """
    _ensure_registered()
    return torch.ops.vlak.fused_attention(
        q, k, v, -1.0 if scale is None else scale, attn_mask,
        -1 if prefix_len is None else prefix_len)


def fused_attention_gqa_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               lengths: torch.Tensor,
                               scale: float | None = None) -> torch.Tensor:
    """GQA attention with per-sample lengths: q (B, M, H, 64), k/v
    (B, N, H_kv, 64) bf16 at any strides, lengths (B,) int32/int64 on the
    device. visible(r, c) = c < L_b and r < L_b (L_b clamped to [0, N]);
    rows r >= L_b are exact zeros. Returns (B, M, H, 64) contiguous."""
    _ensure_registered()
    return torch.ops.vlak.fused_attention_gqa_varlen(
        q, k, v, lengths, -1.0 if scale is None else scale)


def fused_attention_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        scale: float | None = None,
                        prefix_len: int | None = None,
                        dead_start: int = 0,
                        dead_end: int = 0) -> torch.Tensor:
    """Attention where H query heads share H_kv key/value heads.

    Inputs stay in the layout the projections produce: queries (B, M, H, 64)
    and keys / values (B, N, H_kv, 64), bf16, read in place at whatever
    strides they have (head_dim must be the unit-stride dim). Query head h
    uses kv head h // (H // H_kv). No mask tensor: key c is visible to query
    row r when c < prefix_len and c lies outside [dead_start, dead_end), or
    when c >= prefix_len and c <= (N - M) + r (a causal staircase over the
    trailing keys). prefix_len defaults to N and scale to 1/8.

    The result is a new contiguous (B, M, H, 64) tensor, so flattening the
    heads is a free view. A row that sees no key at all comes back as zeros.
    """
    _ensure_registered()
    return torch.ops.vlak.fused_attention_gqa(
        q, k, v, -1.0 if scale is None else scale,
        -1 if prefix_len is None else prefix_len, dead_start, dead_end)


def fused_attention_gqa_v4(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           scale: float | None = None,
                           prefix_len: int | None = None,
                           dead_start: int = 0,
                           dead_end: int = 0) -> torch.Tensor:
    """The reference's v4 entry point; same contract as fused_attention_gqa."""
    _ensure_registered_v4()
    return torch.ops.vlak.fused_attention_gqa_v4(
        q, k, v, -1.0 if scale is None else scale,
        -1 if prefix_len is None else prefix_len, dead_start, dead_end)


def device_error() -> int:
    """Synchronous check of the bounded device waits: waits for the device,
    then reads and clears the error words. Returns the status code of a wait
    that ran out since the last check (5, VLAK_ERR_DEVICE_TIMEOUT), else 0.

    Each op also reads the host-mapped error word on entry, without any
    synchronization, and raises RuntimeError when a kernel that has finished
    since the previous op gave up a wait; this call is for callers that want
    to know at a point of their choosing (e.g. after replaying a CUDA graph,
    whose replays run no host code)."""
    _native.load_ops()
    return int(torch.ops.vlak.device_error())


def check_device_error() -> None:
    """device_error(), raising RuntimeError when a wait ran out."""
    code = device_error()
    if code != 0:
        raise RuntimeError(f"vlak: a kernel gave up a bounded device wait (status {code}); "
                           "the output of that call is incomplete")
