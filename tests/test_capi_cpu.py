"""The C ABI library without a GPU: it loads, exports every symbol the public
header declares, and its host-side validation mirrors the reference's
TORCH_CHECKs (fused_attention.cu:606-633). Nothing here launches a kernel."""
import ctypes
import subprocess

import pytest

from kernels import _native
from tests import capi


def test_library_exports_every_declared_symbol():
    syms = capi.declared_symbols()
    assert len(syms) >= 9
    L = capi.lib()
    for s in syms:
        assert hasattr(L, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", _native.CAPI_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(syms) <= exported
    # nothing but the C ABI is exported
    assert all(e.startswith("vlak_") for e in exported), sorted(exported)


def test_comparator_library_exports_every_declared_symbol():
    syms = capi.declared_symbols(capi.CMP_HEADER, "VLAK_CMP_API")
    assert syms == ["vlak_cmp_last_error_message", "vlak_softmax_cub_fwd",
                    "vlak_softmax_cudnn_fwd"]
    L = _native.comparators()
    for s in syms:
        assert hasattr(L, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", _native.CMP_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(syms)


def test_abi_version_and_status_strings():
    L = capi.lib()
    assert L.vlak_abi_version() == 1
    assert L.vlak_status_string(0) == b"ok"
    assert L.vlak_status_string(5) == b"device-side wait timed out"
    assert L.vlak_status_string(99) == b"unknown status"


@pytest.mark.parametrize("rows,cols", [(1, 16), (31, 100), (32, 100), (32, 2048), (32, 2049),
                                       (4096, 1024), (1, 4096)])
def test_auto_version_matches_reference_rule(rows, cols):
    import torch
    from kernels.softmax import _auto_version

    want = _auto_version(torch.empty(rows, cols))
    assert capi.lib().vlak_softmax_auto_version(rows, cols) == want


def _args(B=1, M=50, N=241, H=15, Hkv=5, P=241, ds=196, de=240, strides=None, base=0x1000):
    a = capi.GqaArgs()
    a.q = a.k = a.v = a.o = base
    a.B, a.M, a.N, a.H, a.Hkv = B, M, N, H, Hkv
    st = strides or [(M * H * 64, H * 64, 64), (N * Hkv * 64, Hkv * 64, 64),
                     (N * Hkv * 64, Hkv * 64, 64), (M * H * 64, H * 64, 64)]
    for name, s in zip(("q_stride", "k_stride", "v_stride", "o_stride"), st):
        arr = getattr(a, name)
        for i in range(3):
            arr[i] = s[i]
    a.scale = -1.0
    a.prefix_len, a.dead_start, a.dead_end = P, ds, de
    return a


def _check(a):
    P = ctypes.c_int64(-7)
    sc = ctypes.c_float(-7)
    st = capi.lib().vlak_attn_gqa_check(ctypes.byref(a), ctypes.byref(P), ctypes.byref(sc))
    return st, P.value, sc.value


def test_check_accepts_the_smolvla_sites_and_resolves_defaults():
    assert _check(_args())[0] == capi.VLAK_OK
    st, P, sc = _check(_args(P=-1, ds=0, de=0))
    assert st == capi.VLAK_OK and P == 241 and sc == pytest.approx(0.125)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(H=15, Hkv=4), capi.VLAK_ERR_INVALID_ARGUMENT, "multiple of kv heads"),
    (dict(P=100, ds=90, de=120), capi.VLAK_ERR_INVALID_ARGUMENT, "dead band"),
    (dict(P=300), capi.VLAK_ERR_INVALID_ARGUMENT, "prefix_len exceeds"),
    (dict(ds=5, de=3), capi.VLAK_ERR_INVALID_ARGUMENT, "dead band"),
    (dict(ds=-1, de=3), capi.VLAK_ERR_INVALID_ARGUMENT, "dead band"),
    (dict(H=256, Hkv=1), capi.VLAK_ERR_INVALID_ARGUMENT, "at most 128"),
    (dict(base=0x1008), capi.VLAK_ERR_ALIGNMENT, "16B alignment"),
    (dict(strides=[(50 * 15 * 64, 15 * 64, 60), (241 * 320, 320, 64), (241 * 320, 320, 64),
                   (50 * 960, 960, 64)]), capi.VLAK_ERR_ALIGNMENT, "16B alignment"),
])
def test_check_rejects_like_the_reference(kw, code, msg):
    st, _, _ = _check(_args(**kw))
    assert st == code
    assert msg in capi.last_error()


def test_empty_problems_are_no_ops_without_a_device():
    L = capi.lib()
    a = _args(B=0)
    assert L.vlak_attn_gqa_fwd(ctypes.byref(a), None) == capi.VLAK_OK
    a = _args(M=0)
    assert L.vlak_attn_gqa_v4_fwd(ctypes.byref(a), None) == capi.VLAK_OK
    assert L.vlak_softmax_fwd(None, None, 0, 5, 0, 4, None) == capi.VLAK_OK
    assert L.vlak_softmax_fwd(None, None, 5, 0, 2, 1, None) == capi.VLAK_OK


def test_softmax_argument_errors():
    L = capi.lib()
    assert L.vlak_softmax_fwd(None, None, -1, 5, 0, 4, None) == capi.VLAK_ERR_INVALID_ARGUMENT
    assert L.vlak_softmax_fwd(0x1000, 0x2000, 4, 5, 7, 4, None) == capi.VLAK_ERR_UNSUPPORTED_DTYPE
    assert L.vlak_softmax_fwd(0x1001, 0x2000, 4, 5, 0, 4, None) == capi.VLAK_ERR_ALIGNMENT
    assert L.vlak_softmax_fwd(None, 0x2000, 4, 5, 0, 4, None) == capi.VLAK_ERR_INVALID_ARGUMENT
