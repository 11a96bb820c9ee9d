"""Build the in-tree CUDA library ``libfp8attn.so`` (sm_100a) with nvcc.

The library is self-contained (static cudart, driver entry points resolved at run time), so it
loads on a machine without a GPU and is shipped beside this file.

    python my-nano-vllm_b200/nanovllm_b200/build.py   # build if any source is newer than the library

(run as a script: importing the package loads the library it builds)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                     # my-nano-vllm_b200/
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB_PATH = os.path.join(PKG_DIR, "libfp8attn.so")

SOURCES = ["capi.cu", "store.cu", "decode.cu", "prefill.cu", "prefill_persistent.cu", "diag.cu",
           "qknorm.cu", "fp8linear.cu"]
HEADERS = ["common.cuh", "kernels.h", "tcgen05.cuh", "prefill_common.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: cannot build libfp8attn.so")
    return cand


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, s) for s in SOURCES]
    files += [os.path.join(CSRC, h) for h in HEADERS if os.path.exists(os.path.join(CSRC, h))]
    files.append(os.path.join(INCLUDE, "fp8attn.h"))
    return files


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if needed; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB_PATH + ".tmp"
    cmd += ["-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
