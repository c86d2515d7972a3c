"""Build libsage_sm100.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/sage_abi.cu includes the kernel headers), built
into tribench_b200/_lib/ so that it travels with the source tree. ``python -m
tribench_b200._build`` rebuilds it; ``build_library()`` rebuilds only when a source file is
newer than the library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libsage_sm100.so")
# the tcgen05 throughput microbenchmark (include/sm100_peaks.h), a library of its own
PEAKS_LIB_PATH = os.path.join(LIB_DIR, "libsm100_peaks.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: cannot build libsage_sm100.so")


def _sources() -> list[str]:
    srcs = glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(CSRC, "sage_abi.cu")]
    srcs.append(os.path.join(ROOT_DIR, "include", "sage_sm100.h"))
    return srcs


def _peaks_sources() -> list[str]:
    return [os.path.join(CSRC, "tensor_peaks.cu"), os.path.join(CSRC, "sm100_ptx.cuh"),
            os.path.join(ROOT_DIR, "include", "sm100_peaks.h")]


def _stale(lib: str, sources: list[str]) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(s) > t for s in sources)


def is_stale() -> bool:
    return _stale(LIB_PATH, _sources())


def _compile(source: str, lib: str, verbose: bool) -> None:
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = lib + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, source]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)


def build_library(force: bool = False, verbose: bool = False) -> str:
    if force or is_stale():
        _compile(os.path.join(CSRC, "sage_abi.cu"), LIB_PATH, verbose)
    return LIB_PATH


def build_peaks_library(force: bool = False, verbose: bool = False) -> str:
    if force or _stale(PEAKS_LIB_PATH, _peaks_sources()):
        _compile(os.path.join(CSRC, "tensor_peaks.cu"), PEAKS_LIB_PATH, verbose)
    return PEAKS_LIB_PATH


if __name__ == "__main__":
    print(build_library(force=True, verbose="-v" in sys.argv))
    print(build_peaks_library(force=True, verbose="-v" in sys.argv))
