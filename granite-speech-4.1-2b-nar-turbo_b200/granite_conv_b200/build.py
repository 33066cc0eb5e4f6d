"""Ahead-of-time build of libgsn_conv.so for sm_100a with nvcc (no JIT, no NVRTC at run time).

    python -m granite_conv_b200.build          # from the package's parent folder

The library is one translation unit (``csrc/gsn_conv_lib.cu``) linked against the static CUDA runtime; the TMA
descriptor encoder comes from the driver at run time through ``cudaGetDriverEntryPoint``, so the library needs
no ``-lcuda``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)                         # granite-speech-4.1-2b-nar-turbo_b200/
REPO_DIR = os.path.dirname(ROOT_DIR)
CSRC = os.path.join(ROOT_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgsn_conv.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + [os.path.join(INCLUDE, "gsn_conv.h")]
    return any(os.path.getmtime(s) > t for s in deps if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/ into lib/libgsn_conv.so (in-tree) and return its path."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I" + CSRC, "-I" + INCLUDE, "-o", tmp, os.path.join(CSRC, "gsn_conv_lib.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
