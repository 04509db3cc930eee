"""Location and loading of the prebuilt native libraries.

``lib/libvlak_b200.so`` holds the CUDA kernels and the C ABI;
``lib/libvlak_torch.so`` registers the ``torch.ops.vlak`` schemas on top of it.
Both are built ahead of time (``python vla-kernels_b200/build.py``); there is no
CPU fallback, so a missing library is an error.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(PKG_ROOT, "lib")
CAPI_PATH = os.path.join(LIB_DIR, "libvlak_b200.so")
TORCH_PATH = os.path.join(LIB_DIR, "libvlak_torch.so")
CMP_PATH = os.path.join(LIB_DIR, "libvlak_comparators.so")

_lock = threading.Lock()
_ops_loaded = False
_capi = None
_cmp = None


def _require(path: str) -> None:
    if not os.path.exists(path):
        raise RuntimeError(
            f"vlak native library missing: {path}. Build it with "
            f"`python {os.path.join(PKG_ROOT, 'build.py')}` (nvcc, sm_100a).")


def load_ops() -> None:
    """Register the torch.ops.vlak schemas (idempotent)."""
    global _ops_loaded
    if _ops_loaded:
        return
    with _lock:
        if not _ops_loaded:
            _require(CAPI_PATH)
            _require(TORCH_PATH)
            torch.ops.load_library(TORCH_PATH)
            _ops_loaded = True


def capi() -> ctypes.CDLL:
    """The C ABI library (include/vlak_b200.h) through ctypes."""
    global _capi
    if _capi is None:
        with _lock:
            if _capi is None:
                _require(CAPI_PATH)
                lib = ctypes.CDLL(CAPI_PATH)
                lib.vlak_status_string.restype = ctypes.c_char_p
                lib.vlak_last_error_message.restype = ctypes.c_char_p
                _capi = lib
    return _capi


def comparators() -> ctypes.CDLL:
    """The softmax comparator library (include/vlak_comparators.h: cuDNN and
    CUB row softmax, benchmark bars) through ctypes."""
    global _cmp
    if _cmp is None:
        with _lock:
            if _cmp is None:
                _require(CMP_PATH)
                lib = ctypes.CDLL(CMP_PATH)
                lib.vlak_cmp_last_error_message.restype = ctypes.c_char_p
                for f in ("vlak_softmax_cudnn_fwd", "vlak_softmax_cub_fwd"):
                    getattr(lib, f).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
                _cmp = lib
    return _cmp
