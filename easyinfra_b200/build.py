"""Build libb200moe.so in-tree with nvcc for sm_100a.

The library is a plain shared object (C ABI, see include/b200moe.h); it links the
CUDA runtime statically so it carries no dependency on the CUDA runtime version
bundled with PyTorch.  Usage: ``python -m easyinfra_b200.build [--verbose]``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libb200moe.so")
SOURCES = ["router.cu", "permute.cu", "norm.cu", "grouped_gemm.cu", "grouped_gemm_wm.cu", "grouped_gemm_2sm.cu", "grouped_gemm_f32.cu", "ep_nvlink.cu", "capi.cu"]
HEADERS = ["ptx.cuh", "common.cuh", "kernels.cuh", "norm_row.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO_DIR, "include", "b200moe.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile the extension if any source is newer than the library; return its path."""
    if not force and not _stale():
        return LIB_PATH
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-cudart",
        "static",
        "-I",
        os.path.join(REPO_DIR, "include"),
        "-o",
        LIB_PATH + ".tmp",
    ]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
