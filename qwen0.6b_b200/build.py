"""Build the native pieces of the package in place.

* ``libqwen_b200.so``: every CUDA kernel plus the C ABI of ``include/*.h``,
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* ``qwen_megakernel_C``, ``rmsnorm``, ``swiglu_fused``: thin PyTorch extension
  modules with the upstream Python-facing operator APIs, linked against
  ``libqwen_b200.so`` (rpath ``$ORIGIN``).

Everything is written next to this file, so the built ``.so`` files travel
with a snapshot of the repository.  Rebuilds are mtime-based.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libqwen_b200.so")
GENCODE = "-gencode=arch=compute_100a,code=sm_100a"
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", GENCODE, "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr"]

# Python extension modules: name -> C++ sources (in csrc/).
EXTENSIONS = {
    "qwen_megakernel_C": ["qwen_ops.cpp"],
    "rmsnorm": ["rmsnorm_ops.cpp"],
    "swiglu_fused": ["swiglu_ops.cpp"],
}


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _newest(paths) -> float:
    return max(os.path.getmtime(p) for p in paths)


def build_native(force: bool = False, verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = (srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest(deps):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, *srcs, "-o", tmp]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def use_system_host_compiler() -> None:
    """Build torch extensions with the system g++/gcc.  The image's CXX / CC
    point at a GCC wrapper that links its own static C++ runtime; an extension
    built that way crashes as soon as it formats a number into a C++ stream
    (every TORCH_CHECK message with a size in it), because the stream code
    meets the shared libstdc++ that torch has loaded."""
    for var, path in (("CXX", "/usr/bin/g++"), ("CC", "/usr/bin/gcc")):
        if os.path.exists(path):
            os.environ[var] = path


def build_extension(name: str, force: bool = False, verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in EXTENSIONS[name]]
    dst = os.path.join(PKG, f"{name}.so")
    deps = srcs + [LIB] + glob.glob(os.path.join(INCLUDE, "*.h"))
    if not force and os.path.exists(dst) and os.path.getmtime(dst) >= _newest(deps):
        return dst
    from torch.utils.cpp_extension import load

    use_system_host_compiler()
    workdir = os.path.join(PKG, "_build", name)
    os.makedirs(workdir, exist_ok=True)
    load(
        name=name,
        sources=srcs,
        extra_include_paths=[INCLUDE, CSRC],
        extra_cflags=["-O2"],
        # "$$" survives ninja, the single quotes survive /bin/sh: the linker
        # sees the literal $ORIGIN.
        extra_ldflags=[f"-L{PKG}", "-lqwen_b200", "-Wl,-rpath,'$$ORIGIN:$$ORIGIN/../..'"],
        build_directory=workdir,
        with_cuda=True,
        is_python_module=True,
        verbose=verbose,
    )
    shutil.copy2(os.path.join(workdir, f"{name}.so"), dst)
    return dst


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_native(force=force, verbose=verbose)
    for name in EXTENSIONS:
        build_extension(name, force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
