"""Rebuild the reference's own CUDA kernels for sm_100a, as benchmark bars.

The reference (djkim9031-research/vla-kernels) JIT-builds its kernels for the
local GPU with ``-arch=native`` (kernels/softmax/__init__.py:40-53,
kernels/attention/__init__.py:17-31, :50-60). This recipe compiles the same
source files, unmodified and read in place from a checkout, for B200
(``-gencode arch=compute_100a,code=sm_100a``, the reference's other flags
kept: ``-O3 --use_fast_math``). Nothing is copied into this repository; the
built libraries go to ``baseline/_ref/kernels_sm100a/`` (git-ignored; they
travel to the GPU box with the working tree).

  python baseline/build_ref_kernels.py --reference PATH   (or VLAK_REFERENCE=PATH)

Built: vlak_ref_softmax (softmax_kernels.cu: versions 0-4), vlak_ref_attention
(fused_attention.cu: v1/v2 and the v3 GQA kernel), and vlak_ref_attention_v4
(fused_attention_v4.cu, CuTe SM80 mma.sync atoms) when CuTe headers are found
(the reference's own third_party/cutlass submodule is empty in its checkout;
the recipe takes CUTLASS_HOME, else the CUTLASS tree vendored by the
flashinfer wheel). Each library registers the reference's torch.ops.vlak
schemas, so it must not be loaded into a process that also loads this
package's libvlak_torch.so: bench.py loads them in a separate process.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "kernels_sm100a")
FLAGS = ["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"]


def _cutlass_include() -> str | None:
    cand = os.environ.get("CUTLASS_HOME")
    if cand and os.path.isdir(os.path.join(cand, "include", "cute")):
        return os.path.join(cand, "include")
    try:
        import flashinfer  # noqa: F401  (only for the location of its CUTLASS tree)
        root = os.path.dirname(flashinfer.__file__)
    except Exception:
        import importlib.util
        spec = importlib.util.find_spec("flashinfer")
        root = os.path.dirname(spec.origin) if spec and spec.origin else None
    if root:
        inc = os.path.join(root, "data", "cutlass", "include")
        if os.path.isdir(os.path.join(inc, "cute")):
            return inc
    return None


def build(reference: str) -> dict:
    from torch.utils.cpp_extension import load

    os.makedirs(OUT, exist_ok=True)
    jobs = [
        ("vlak_ref_softmax", "kernels/softmax/softmax_kernels.cu", []),
        ("vlak_ref_attention", "kernels/attention/fused_attention.cu", []),
    ]
    cutlass = _cutlass_include()
    if cutlass:
        jobs.append(("vlak_ref_attention_v4", "kernels/attention/fused_attention_v4.cu", [cutlass]))
    status = {}
    for name, rel, incs in jobs:
        d = os.path.join(OUT, name)
        os.makedirs(d, exist_ok=True)
        try:
            load(name=name, sources=[os.path.join(reference, rel)], extra_include_paths=incs,
                 extra_cuda_cflags=FLAGS, build_directory=d, is_python_module=False,
                 verbose=False)
            status[name] = {"source": rel, "so": os.path.join(name, f"{name}.so"), "ok": True}
        except Exception as e:  # a comparator that does not build is reported, not fatal
            status[name] = {"source": rel, "ok": False, "error": str(e).splitlines()[-1][:300]}
    if not cutlass:
        status["vlak_ref_attention_v4"] = {"source": "kernels/attention/fused_attention_v4.cu",
                                           "ok": False, "error": "no CuTe headers found"}
    with open(os.path.join(OUT, "manifest.json"), "w") as f:
        json.dump(status, f, indent=1)
    return status


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VLAK_REFERENCE"))
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(os.path.join(a.reference, "kernels")):
        ap.error("give the reference checkout with --reference PATH or VLAK_REFERENCE=PATH")
    print(json.dumps(build(a.reference), indent=1))


if __name__ == "__main__":
    sys.exit(main())
