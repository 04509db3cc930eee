"""ctypes view of the C ABI (include/vlak_b200.h) for the tests.

The GPU parity tests call the kernels through these entry points with device
pointers of torch tensors, exactly as a non-torch host would.
"""
from __future__ import annotations

import ctypes
import re
import os

import torch

from kernels import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "vlak_b200.h")

VLAK_OK = 0
VLAK_ERR_INVALID_ARGUMENT = 1
VLAK_ERR_ALIGNMENT = 2
VLAK_ERR_UNSUPPORTED_DTYPE = 3
VLAK_ERR_DEVICE_TIMEOUT = 5
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


class GqaArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("B", ctypes.c_int64), ("M", ctypes.c_int64), ("N", ctypes.c_int64),
        ("H", ctypes.c_int64), ("Hkv", ctypes.c_int64),
        ("q_stride", ctypes.c_int64 * 3), ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3), ("o_stride", ctypes.c_int64 * 3),
        ("scale", ctypes.c_double),
        ("prefix_len", ctypes.c_int64), ("dead_start", ctypes.c_int64),
        ("dead_end", ctypes.c_int64),
    ]


def lib():
    L = _native.capi()
    L.vlak_softmax_fwd.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.vlak_softmax_auto_version.argtypes = [ctypes.c_int64, ctypes.c_int64]
    for f in ("vlak_attn_gqa_fwd", "vlak_attn_gqa_v4_fwd"):
        getattr(L, f).argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p]
    L.vlak_attn_gqa_check.argtypes = [ctypes.POINTER(GqaArgs), ctypes.POINTER(ctypes.c_int64),
                                      ctypes.POINTER(ctypes.c_float)]
    L.vlak_device_error_read.argtypes = [ctypes.POINTER(ctypes.c_int)]
    L.vlak_device_error_poll.argtypes = [ctypes.POINTER(ctypes.c_int)]
    L.vlak_attn_gqa_workspace_size.argtypes = [ctypes.POINTER(GqaArgs), ctypes.POINTER(ctypes.c_int64)]
    L.vlak_attn_gqa_fwd_ws.argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_void_p]
    L.vlak_attn_gqa_varlen_fwd.argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p, ctypes.c_int,
                                           ctypes.c_void_p]
    L.vlak_attn_gqa_varlen_fwd_ws.argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p,
                                              ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_void_p]
    L.vlak_attn_gqa_masked_fwd.argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    L.vlak_attn_gqa_masked_fwd_ws.argtypes = [ctypes.POINTER(GqaArgs), ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_void_p]
    L.vlak_selftest_wait_timeout.argtypes = [ctypes.c_void_p]
    return L


CMP_HEADER = os.path.join(os.path.dirname(HEADER), "vlak_comparators.h")


def declared_symbols(header: str = HEADER, macro: str = "VLAK_API") -> list[str]:
    """Every function a public header declares."""
    text = open(header).read()
    return sorted(set(re.findall(macro + r"\s+[\w\s\*]+?\b(vlak_\w+)\s*\(", text)))


def gqa_args(q, k, v, o, prefix_len=-1, dead_start=0, dead_end=0, scale=-1.0,
             shape=None, strides=None) -> GqaArgs:
    a = GqaArgs()
    a.q, a.k, a.v = q.data_ptr() if q is not None else 0, k.data_ptr() if k is not None else 0, \
        v.data_ptr() if v is not None else 0
    a.o = o.data_ptr() if o is not None else 0
    if shape is None:
        B, M, H, _ = q.shape
        N, Hkv = k.shape[1], k.shape[2]
    else:
        B, M, N, H, Hkv = shape
    a.B, a.M, a.N, a.H, a.Hkv = B, M, N, H, Hkv
    if strides is None:
        strides = [t.stride()[:3] if t is not None else (0, 0, 0) for t in (q, k, v, o)]
    for name, st in zip(("q_stride", "k_stride", "v_stride", "o_stride"), strides):
        arr = getattr(a, name)
        for i in range(3):
            arr[i] = st[i]
    a.scale = scale
    a.prefix_len, a.dead_start, a.dead_end = prefix_len, dead_start, dead_end
    return a


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def attn_gqa(q, k, v, prefix_len=-1, dead_start=0, dead_end=0, scale=-1.0, v4=False):
    """Run the GQA kernel through the C ABI; returns (status, o)."""
    L = lib()
    B, M, H, D = q.shape
    o = torch.empty(B, M, H, D, device=q.device, dtype=torch.bfloat16)
    a = gqa_args(q, k, v, o, prefix_len, dead_start, dead_end, scale)
    f = L.vlak_attn_gqa_v4_fwd if v4 else L.vlak_attn_gqa_fwd
    st = f(ctypes.byref(a), stream_ptr())
    return st, o


def workspace_size(q, k, v, prefix_len=-1, dead_start=0, dead_end=0) -> int:
    """Bytes the key-split (_ws) entry points want for these arguments."""
    B, M, H, D = q.shape
    o = torch.empty(B, M, H, D, device=q.device, dtype=torch.bfloat16)
    a = gqa_args(q, k, v, o, prefix_len, dead_start, dead_end)
    n = ctypes.c_int64(-1)
    st = lib().vlak_attn_gqa_workspace_size(ctypes.byref(a), ctypes.byref(n))
    assert st == VLAK_OK, last_error()
    return n.value


def attn_gqa_ws(q, k, v, prefix_len=-1, dead_start=0, dead_end=0, scale=-1.0, lengths=None,
                mask=None, workspace=None):
    """Run the GQA kernel through a key-split (_ws) entry point with a
    workspace of the size the library asks for (or the given one); lengths
    selects the varlen form, mask (B, M, N bool) the masked form. Returns
    (status, o)."""
    L = lib()
    B, M, H, D = q.shape
    o = torch.empty(B, M, H, D, device=q.device, dtype=torch.bfloat16)
    a = gqa_args(q, k, v, o, prefix_len, dead_start, dead_end, scale)
    if workspace is None:
        n = ctypes.c_int64(0)
        assert L.vlak_attn_gqa_workspace_size(ctypes.byref(a), ctypes.byref(n)) == VLAK_OK
        workspace = torch.empty(max(n.value, 1), device=q.device, dtype=torch.uint8)
    wp, wn = workspace.data_ptr(), workspace.numel()
    if lengths is not None:
        dt = 5 if lengths.dtype == torch.int64 else 4
        st = L.vlak_attn_gqa_varlen_fwd_ws(ctypes.byref(a), lengths.data_ptr(), dt, wp, wn,
                                           stream_ptr())
    elif mask is not None:
        N = k.shape[1]
        st = L.vlak_attn_gqa_masked_fwd_ws(ctypes.byref(a), mask.data_ptr(), M * N, N, wp, wn,
                                           stream_ptr())
    else:
        st = L.vlak_attn_gqa_fwd_ws(ctypes.byref(a), wp, wn, stream_ptr())
    return st, o


def attn_gqa_plain(q, k, v, lengths=None, mask=None, prefix_len=-1, dead_start=0, dead_end=0):
    """The unsplit entry points (varlen / masked / analytic)."""
    L = lib()
    B, M, H, D = q.shape
    o = torch.empty(B, M, H, D, device=q.device, dtype=torch.bfloat16)
    a = gqa_args(q, k, v, o, prefix_len, dead_start, dead_end)
    if lengths is not None:
        dt = 5 if lengths.dtype == torch.int64 else 4
        st = L.vlak_attn_gqa_varlen_fwd(ctypes.byref(a), lengths.data_ptr(), dt, stream_ptr())
    elif mask is not None:
        N = k.shape[1]
        st = L.vlak_attn_gqa_masked_fwd(ctypes.byref(a), mask.data_ptr(), M * N, N, stream_ptr())
    else:
        st = L.vlak_attn_gqa_fwd(ctypes.byref(a), stream_ptr())
    return st, o


def softmax(x, version=4):
    L = lib()
    y = torch.empty_like(x)
    st = L.vlak_softmax_fwd(x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1],
                            DTYPES[x.dtype], version, stream_ptr())
    return st, y


def last_error() -> str:
    return (lib().vlak_last_error_message() or b"").decode()
