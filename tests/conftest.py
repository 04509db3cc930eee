"""pytest configuration: the `gpu` marker, import paths, native build."""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "vla-kernels_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _ensure_built():
    lib = os.path.join(PKG, "lib")
    if not (os.path.exists(os.path.join(lib, "libvlak_b200.so"))
            and os.path.exists(os.path.join(lib, "libvlak_torch.so"))):
        import build  # vla-kernels_b200/build.py
        build.build_all()


_ensure_built()


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
