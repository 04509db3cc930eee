"""The Python boundary without a GPU: the operator schemas are byte-identical
to the reference's, the fake (meta) implementations shape-infer, and the
wrapper API (versions, routing, register guards) is the reference's."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from kernels import attention, softmax as sm

# kernels/softmax/softmax_kernels.cu:303-305, fused_attention.cu:671-676,
# fused_attention_v4.cu:333-336
REF_SCHEMAS = {
    "softmax": "vlak::softmax(Tensor x, int version=4) -> Tensor",
    "fused_attention_gqa": "vlak::fused_attention_gqa(Tensor q, Tensor k, Tensor v, "
                           "float scale=-1., int prefix_len=-1, int dead_start=0, "
                           "int dead_end=0) -> Tensor",
    "fused_attention_gqa_v4": "vlak::fused_attention_gqa_v4(Tensor q, Tensor k, Tensor v, "
                              "float scale=-1., int prefix_len=-1, int dead_start=0, "
                              "int dead_end=0) -> Tensor",
}


@pytest.fixture(scope="module", autouse=True)
def registered():
    sm._ext()
    attention._ext()
    attention._ext_v4()


@pytest.mark.parametrize("name", list(REF_SCHEMAS))
def test_schema_is_the_reference_schema(name):
    op = getattr(torch.ops.vlak, name).default
    assert str(op._schema) == REF_SCHEMAS[name]


def test_only_cuda_kernels_are_registered():
    # no CPU fallback: the op has a CUDA kernel and a Meta (fake) impl only
    for name in REF_SCHEMAS:
        assert torch._C._dispatch_has_kernel_for_dispatch_key(f"vlak::{name}", "CUDA")
        assert not torch._C._dispatch_has_kernel_for_dispatch_key(f"vlak::{name}", "CPU")


def test_softmax_versions_and_best():
    assert sm.VERSIONS == {"v0": 0, "v1": 1, "v2": 2, "v3": 3, "v4": 4}
    assert sm.BEST == "auto"


@pytest.mark.parametrize("shape,want", [((4096, 1024), 1), ((8, 1024), 4), ((32, 2049), 4),
                                        ((983040, 291), 1), ((64, 16384), 4)])
def test_auto_version(shape, want):
    assert sm._auto_version(torch.empty(*shape)) == want


def test_softmax_fake_is_contiguous_same_shape():
    with FakeTensorMode():
        x = torch.empty(8, 64, device="cuda", dtype=torch.bfloat16)
        y = torch.ops.vlak.softmax(x, 4)
    assert y.shape == (8, 64) and y.dtype == torch.bfloat16 and y.is_contiguous()


@pytest.mark.parametrize("fn", ["fused_attention_gqa", "fused_attention_gqa_v4"])
def test_attention_fake_promises_contiguous_q_shape(fn):
    with FakeTensorMode():
        qb = torch.empty(2, 50, 17, 64, device="cuda", dtype=torch.bfloat16)
        q = qb[:, :, 1:16]
        k = torch.empty(2, 291, 5, 64, device="cuda", dtype=torch.bfloat16)
        o = getattr(torch.ops.vlak, fn)(q, k, k, -1.0, 241, 196, 240)
    assert o.shape == (2, 50, 15, 64) and o.is_contiguous()


def test_unknown_version_name_raises_keyerror():
    with pytest.raises(KeyError):
        sm.softmax(torch.empty(2, 2), "v9")


def test_register_guards_are_plain_bools():
    # Dynamo folds a module-level bool; lru_cache would graph-break
    assert sm._registered is True or sm._registered is False
    sm._ensure_registered()
    assert sm._registered is True
    attention._ensure_registered()
    attention._ensure_registered_v4()
    assert attention._registered and attention._registered_v4
