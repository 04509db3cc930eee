"""Fused row-softmax on B200 (sm_100a), registered as ``vlak::softmax``.

Same API as the reference module (kernels/softmax/__init__.py): ``softmax``,
``VERSIONS``, ``BEST``, ``_auto_version``, ``_ext`` and the fake (meta)
implementation, so callers such as ``vla/patch_kernels.py`` work unchanged and
the op traces as a single node under ``torch.compile(fullgraph=True)``.

The kernels are prebuilt for sm_100a (lib/libvlak_b200.so); the versions
select the same algorithm families as the reference ladder, re-designed for
B200 (see vla-kernels_b200/csrc/softmax.cu).
"""
from __future__ import annotations

from functools import lru_cache

import torch

from .. import _native

# softmax version names -> int passed to the kernel dispatcher
VERSIONS = {"v0": 0, "v1": 1, "v2": 2, "v3": 3, "v4": 4}
BEST = "auto"


def _auto_version(x: torch.Tensor) -> int:
    # kernels/softmax/__init__.py:26-37: wide rows -> v4, many narrow rows ->
    # v1 (warp per row), few rows -> v4 (block per row)
    rows, cols = x.shape
    if cols > 2048:
        return VERSIONS["v4"]
    if rows >= 32:
        return VERSIONS["v1"]
    return VERSIONS["v4"]


@lru_cache(maxsize=1)
def _ext():
    _native.load_ops()
    # loading the library ran TORCH_LIBRARY(vlak); the fake (meta) impl lets
    # FakeTensor tracing shape-infer the op, promising a contiguous output
    torch.library.register_fake("vlak::softmax")(
        lambda x, version=4: torch.empty(x.shape, dtype=x.dtype, device=x.device))
    return torch.ops.vlak


_registered = False


def _ensure_registered():
    # plain global-bool guard so Dynamo folds this branch instead of breaking
    global _registered
    if not _registered:
        _ext()
        _registered = True


def softmax(x: torch.Tensor, version: str | int = BEST) -> torch.Tensor:
    """Softmax over the last dim of a 2D ``[rows, cols]`` CUDA tensor.

    Routed through the dispatcher-registered op (vlak::softmax), so calls
    compose with torch.compile / torch.export instead of graph-breaking.
    """
    if version == "auto":
        v = _auto_version(x)
    elif isinstance(version, str):
        v = VERSIONS[version]
    else:
        v = int(version)
    _ensure_registered()
    return torch.ops.vlak.softmax(x, v)


# ---- library comparators (cuDNN softmax, CUB-primitive softmax) -------------
# The reference builds these as a separate extension for benchmarking
# (kernels/softmax/softmax_baselines.cu). They are not part of this build.

def softmax_cudnn(x: torch.Tensor) -> torch.Tensor:
    """Vendor comparator (reference: cudnnSoftmaxForward); not built here."""
    raise RuntimeError("softmax_cudnn comparator is not built in the B200 package")


def softmax_cub(x: torch.Tensor) -> torch.Tensor:
    """Library-primitive comparator (reference: cub::BlockReduce); not built here."""
    raise RuntimeError("softmax_cub comparator is not built in the B200 package")
