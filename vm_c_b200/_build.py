"""Builds the native extensions in-tree.

Two extensions:
  * ``_host``  — C++17 host runtime (GGUF, quant codecs, block manager, scheduler). No CUDA.
  * ``_cuda``  — sm_100a kernels (tcgen05 / TMA GEMMs, attention, norms, sampling, comm) and their
                 launchers. Compiled only for ``sm_100a``; nothing else is generated.

The shared objects land in ``vm_c_b200/_ext/<name>/`` so that they travel with a copy of the
repository; :mod:`vm_c_b200._native` imports them from there without invoking the compiler.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
EXT_DIR = PKG_DIR / "_ext"
CSRC = REPO_DIR / "csrc"

HOST_SOURCES = ["host/gguf.cpp", "host/quants.cpp", "host/block_manager.cpp", "host/scheduler.cpp",
                "host/tokenizer.cpp", "host/turboquant.cpp", "host/safetensors.cpp", "host/bindings.cpp"]

SM100_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a"]


def cuda_sources() -> list[str]:
    kdir = CSRC / "kernels"
    return sorted(str(p) for p in kdir.glob("*.cu")) + sorted(str(p) for p in kdir.glob("*.cpp"))


def _jobs() -> None:
    os.environ.setdefault("MAX_JOBS", str(max(1, min(16, os.cpu_count() or 4))))


def build_host(verbose: bool = False):
    from torch.utils.cpp_extension import load
    _jobs()
    out = EXT_DIR / "host"
    out.mkdir(parents=True, exist_ok=True)
    return load(name="_host", sources=[str(CSRC / s) for s in HOST_SOURCES],
                extra_cflags=["-O3", "-std=c++17", "-fvisibility=hidden", "-Wno-unused-function"],
                extra_include_paths=[str(CSRC / "host")], build_directory=str(out), verbose=verbose,
                is_python_module=True)


def build_cuda(verbose: bool = False):
    from torch.utils.cpp_extension import load
    _jobs()
    out = EXT_DIR / "cuda"
    out.mkdir(parents=True, exist_ok=True)
    cuda_flags = SM100_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                                "-Xptxas=-v" if os.environ.get("VMC_PTXAS_VERBOSE") else "-Xptxas=-O3",
                                "-DNDEBUG", "-U__CUDA_NO_HALF_OPERATORS__",
                                "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                                "-U__CUDA_NO_HALF2_OPERATORS__"] + os.environ.get("VMC_NVCC_EXTRA", "").split()
    return load(name="_cuda", sources=cuda_sources(),
                extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=cuda_flags,
                extra_include_paths=[str(CSRC / "kernels"), str(CSRC / "host")],
                extra_ldflags=["-lcuda"], build_directory=str(out), verbose=verbose,
                is_python_module=True)


def build_all(verbose: bool = False) -> None:
    build_host(verbose)
    build_cuda(verbose)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    v = "-v" in sys.argv
    if what in ("host", "all"):
        build_host(v)
    if what in ("cuda", "all"):
        build_cuda(v)
