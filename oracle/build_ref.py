"""Build recipe for the reference implementation, used only as a test checker.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  This script compiles the upstream
project's own CUDA/C++ sources, unmodified and in place under the read-only
reference checkout, into three Python extension modules written to
``oracle/_ref/`` (git-ignored; the built ``.so`` files travel to the GPU box):

* ``qwen_megakernel_C`` from ``Tools/megakernel/megakernel.cu`` +
  ``Tools/megakernel/qwen_ops.cpp`` (include dirs ``Tools/rmsnorm`` and
  ``Tools/swiglu``, because ``megakernel.cu:7-9`` includes ``rmsnorm.cuh`` and
  ``swiglu.cu``);
* ``rmsnorm`` from ``Tools/rmsnorm/rmsnorm.cu``;
* ``swiglu_fused`` from ``Tools/swiglu/swiglu.cu`` + ``swiglu_binding.cpp``.

The upstream project ships no build file (its ``setup.py`` is git-ignored and
absent, ``.gitignore:5``); the module names come from ``.gitignore:7-9``.
The modules are only ever *run* on a B200 box, by ``tests/golden/make_golden.py``
and the reference-parity GPU tests, to pin the CPU oracle.  Nothing in the
product imports them.

Usage: ``python oracle/build_ref.py [--ref /path/to/reference]``.  When the
reference checkout is absent the script prints a note and exits 0.
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
GENCODE = "-gencode=arch=compute_100a,code=sm_100a"


def _build(name: str, sources: list[str], includes: list[str], workdir: str) -> None:
    from torch.utils.cpp_extension import load

    os.makedirs(workdir, exist_ok=True)
    load(
        name=name,
        sources=sources,
        extra_include_paths=includes,
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", GENCODE],
        build_directory=workdir,
        is_python_module=True,
        verbose=False,
    )
    so = os.path.join(workdir, f"{name}.so")
    if not os.path.exists(so):
        raise RuntimeError(f"reference build produced no {so}")
    shutil.copy2(so, os.path.join(OUT, f"{name}.so"))


def build(ref: str) -> bool:
    if not os.path.isdir(os.path.join(ref, "Tools", "megakernel")):
        print(f"[build_ref] reference checkout not found at {ref}; skipping")
        return False
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    # The image's CXX / CC wrapper links a static C++ runtime that crashes
    # on stream formatting next to torch's shared libstdc++; use the system
    # compilers, as the package build does.
    for var, path in (("CXX", "/usr/bin/g++"), ("CC", "/usr/bin/gcc")):
        if os.path.exists(path):
            os.environ[var] = path
    os.makedirs(OUT, exist_ok=True)
    t = os.path.join(ref, "Tools")
    mk, rn, sw = (os.path.join(t, d) for d in ("megakernel", "rmsnorm", "swiglu"))
    targets = [
        ("qwen_megakernel_C",
         [os.path.join(mk, "megakernel.cu"), os.path.join(mk, "qwen_ops.cpp")], [rn, sw]),
        ("rmsnorm", [os.path.join(rn, "rmsnorm.cu")], [rn]),
        ("swiglu_fused",
         [os.path.join(sw, "swiglu.cu"), os.path.join(sw, "swiglu_binding.cpp")], [sw]),
    ]
    for name, srcs, incs in targets:
        dst = os.path.join(OUT, f"{name}.so")
        newest = max(os.path.getmtime(s) for s in srcs)
        if os.path.exists(dst) and os.path.getmtime(dst) >= newest:
            continue
        print(f"[build_ref] building {name}")
        _build(name, srcs, incs, os.path.join(OUT, "build_" + name))
    return True


def reference_dir() -> str:
    """$QWEN_REFERENCE_DIR, else BASELINE.json's "reference_path" (repo root)."""
    env = os.environ.get("QWEN_REFERENCE_DIR")
    if env:
        return env
    try:
        import json
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            return json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        return ""


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=reference_dir())
    args = ap.parse_args()
    build(args.ref)
    sys.exit(0)
