"""Build the CUDA library in-tree (tinygpt_b200/libtgsample.so) for sm_100a."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtgsample.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# --fmad=false: the sampling semantics are defined op by op; no contraction.
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "--fmad=false",
         "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-diag-suppress", "177,128"]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cuh", ".cpp")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    hdr = os.path.join(HERE, "..", "include", "tgsample.h")
    return any(os.path.getmtime(f) > t for f in sources() + [hdr])


def build(force: bool = False, verbose: bool = False) -> str:
    if force or needs_build():
        cmd = [NVCC, *FLAGS, "-o", LIB, os.path.join(CSRC, "tgsample.cu"),
               os.path.join(CSRC, "tg_grammar.cpp")]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
