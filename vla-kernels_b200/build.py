"""Build the in-tree native libraries of the vla-kernels B200 package.

  lib/libvlak_b200.so   CUDA kernels + the C ABI of include/vlak_b200.h
                        (nvcc, sm_100a only, static cudart, no torch)
  lib/libvlak_torch.so  torch.ops.vlak schema registration calling the C ABI
                        (g++, torch headers / libraries; no CUDA code)
  lib/libvlak_comparators.so
                        library comparators for the softmax benchmark (cuDNN,
                        CUB), C ABI of include/vlak_comparators.h

Both are rebuilt only when a source is newer than the library. Run directly
(``python vla-kernels_b200/build.py [--force]``) or through
``__graft_entry__.build()``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "lib")
INCLUDE = os.path.join(REPO, "include")

CAPI_LIB = os.path.join(LIB_DIR, "libvlak_b200.so")
TORCH_LIB = os.path.join(LIB_DIR, "libvlak_torch.so")
CMP_LIB = os.path.join(LIB_DIR, "libvlak_comparators.so")

CU_SOURCES = ["capi.cu", "softmax.cu", "attention_gqa.cu", "attention_simt.cu"]
HEADERS = ["vlak_device.cuh", "vlak_internal.h"]
SHIM_SOURCES = ["torch_ops.cpp"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    if not os.path.exists(os.path.join(home, "bin", "nvcc")):
        nvcc = shutil.which("nvcc")
        if nvcc is None:
            raise RuntimeError("nvcc not found: set CUDA_HOME")
        home = os.path.dirname(os.path.dirname(nvcc))
    return home


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n"
                           f"{r.stdout}\n{r.stderr}")


def build_capi(force: bool = False, verbose_ptxas: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "vlak_b200.h")]
    if not force and not _stale(CAPI_LIB, deps):
        return CAPI_LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    nvcc = os.path.join(_cuda_home(), "bin", "nvcc")
    cmd = [nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-I", INCLUDE, "-o", CAPI_LIB + ".tmp", *srcs]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd)
    os.replace(CAPI_LIB + ".tmp", CAPI_LIB)
    return CAPI_LIB


def build_torch_shim(force: bool = False) -> str:
    import torch.utils.cpp_extension as cpp

    srcs = [os.path.join(CSRC, s) for s in SHIM_SOURCES]
    deps = srcs + [os.path.join(INCLUDE, "vlak_b200.h"), CAPI_LIB]
    if not force and not _stale(TORCH_LIB, deps):
        return TORCH_LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    import torch

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", INCLUDE, "-I", os.path.join(_cuda_home(), "include")]
    for inc in cpp.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-o", TORCH_LIB + ".tmp", *srcs]
    for libdir in cpp.library_paths():
        cmd += ["-L", libdir, f"-Wl,-rpath,{libdir}"]
    cmd += ["-L", LIB_DIR, "-Wl,-rpath,$ORIGIN", "-lvlak_b200",
            "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch"]
    _run(cmd)
    os.replace(TORCH_LIB + ".tmp", TORCH_LIB)
    return TORCH_LIB


def build_comparators(force: bool = False) -> str:
    src = os.path.join(CSRC, "comparators.cu")
    deps = [src, os.path.join(INCLUDE, "vlak_comparators.h")]
    if not force and not _stale(CMP_LIB, deps):
        return CMP_LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    nvcc = os.path.join(_cuda_home(), "bin", "nvcc")
    cmd = [nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-I", INCLUDE, "-o", CMP_LIB + ".tmp", src, "-lcudnn"]
    _run(cmd)
    os.replace(CMP_LIB + ".tmp", CMP_LIB)
    return CMP_LIB


def build_all(force: bool = False) -> list[str]:
    return [build_capi(force), build_torch_shim(force), build_comparators(force)]


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    if a.ptxas_verbose:
        build_capi(force=True, verbose_ptxas=True)
    for p in build_all(a.force):
        print(p)
    sys.exit(0)
