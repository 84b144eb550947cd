"""Compile ``libsiglip2_b200.so`` in-tree for sm_100a with nvcc.

    python -m siglip2_b200.build          # or __graft_entry__.build()

The library is a single translation unit (``csrc/siglip2_capi.cu``) with a
plain C ABI (``include/siglip2_b200.h``); it links only the CUDA runtime and
reaches the driver's ``cuTensorMapEncodeTiled`` through
``cudaGetDriverEntryPoint``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libsiglip2_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = [os.path.join(HERE, "csrc", "siglip2_capi.cu")]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_source_mtime() -> float:
    t = 0.0
    for root in (os.path.join(HERE, "csrc"), os.path.join(os.path.dirname(HERE), "include")):
        for dp, _, fns in os.walk(root):
            for fn in fns:
                t = max(t, os.path.getmtime(os.path.join(dp, fn)))
    return t


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= _newest_source_mtime():
        return LIB_PATH
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-shared", "-o", LIB_PATH + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
