"""Row softmax oracle (test infrastructure only).

Restates the computation of the reference kernels and of their oracle:
  kernels/softmax/softmax_kernels.cu:36-56 (v1) / :149-205 (v4): row max m in
  fp32, e = exp(x - m) with the difference formed in fp32, s = sum(e),
  y = e / s; tests/test_softmax.py:24-30 checks against
  torch.softmax(x.float()).
Here the fp32 difference is kept (it is what torch and the kernels both
round), and everything after it is float64, so the result is the exact value
of the fp32 pipeline up to one final rounding. A row of all -inf gives NaN,
as torch.softmax does.
"""
from __future__ import annotations

import numpy as np


def softmax_rows(x: np.ndarray) -> np.ndarray:
    """Softmax over the last axis of a 2D array; returns float64."""
    x32 = np.asarray(x, dtype=np.float32)
    if x32.ndim != 2:
        raise ValueError("expected a 2D [rows, cols] array")
    with np.errstate(invalid="ignore", over="ignore"):
        m = x32.max(axis=1, keepdims=True) if x32.shape[1] else np.zeros((x32.shape[0], 1), np.float32)
        d = (x32 - m).astype(np.float32)          # the fp32 subtraction
        e = np.exp(d.astype(np.float64))
        s = e.sum(axis=1, keepdims=True)
        y = e / s
    return y


def softmax_rows_torch_cpu(x, threads: int | None = None):
    """The reference's CPU path (torch.softmax on host cores), for timing.

    ``x`` is a CPU torch tensor; math is fp32 as in the reference's tests.
    """
    import torch

    if threads:
        torch.set_num_threads(threads)
    return torch.softmax(x.float(), dim=-1).to(x.dtype)
