"""Builds the CUDA library ``autoindexer_b200/_ai_attn.so`` in-tree for sm_100a.

``python -m autoindexer_b200.build`` (or ``build()``) runs nvcc on the
sources in ``autoindexer_b200/csrc``; the library exports the C ABI of
``include/ai_attn.h``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_ai_attn.so")
SOURCES = ["ai_capi.cu", "ai_attn_simt.cu", "ai_attn_fwd_sm100.cu", "ai_attn_bwd_sm100.cu", "ai_prerot.cu",
           "ai_noalloc.cu", "ai_profile.cu", "ai_decode.cu", "ai_selftest.cu", "ai_index.cu", "ai_prep.cpp"]
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "ai_attn.h"))
    if not force and os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps):
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *FLAGS, "-o", tmp, *srcs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
