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
# Benchmark bars, as in the reference (kernels/softmax/__init__.py:78-114,
# kernels/softmax/softmax_baselines.cu): not the product path, and not
# dispatcher ops. They run from lib/libvlak_comparators.so on the current
# stream.

_CMP_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _comparator(fn_name: str, x: torch.Tensor) -> torch.Tensor:
    import ctypes

    if not x.is_cuda or x.dim() != 2:
        raise RuntimeError("expected a 2D [rows, cols] CUDA tensor")
    if x.dtype not in _CMP_DTYPES:
        raise RuntimeError(f"unsupported dtype {x.dtype}")
    lib = _native.comparators()
    with torch.cuda.device(x.device):
        x = x.contiguous()
        y = torch.empty_like(x)
        st = getattr(lib, fn_name)(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                   x.shape[0], x.shape[1], _CMP_DTYPES[x.dtype],
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if st != 0:
        raise RuntimeError(f"{fn_name}: {lib.vlak_cmp_last_error_message().decode()} (status {st})")
    return y


def softmax_cudnn(x: torch.Tensor) -> torch.Tensor:
    """Vendor comparator: cudnnSoftmaxForward (accurate, per row)."""
    return _comparator("vlak_softmax_cudnn_fwd", x)


def softmax_cub(x: torch.Tensor) -> torch.Tensor:
    """Library-primitive comparator: block per row, cub::BlockReduce max/sum."""
    return _comparator("vlak_softmax_cub_fwd", x)
