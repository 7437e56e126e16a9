"""Build libmockbird_kv.so in-tree with nvcc for sm_100a.

    python -m mockbird_b200.build          # or: __graft_entry__.build()

The library is plain CUDA C++ behind the C ABI of include/mockbird_kv.h; it
does not link against torch.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmockbird_kv.so")

SOURCES = ["mb_api.cu", "mb_decode.cu", "mb_decode_persist.cu", "mb_prefill.cu", "mb_prefill_tc.cu", "mb_gemm.cu",
           "mb_decoder.cu", "mb_local.cu", "mb_noalloc.cu"]
HEADERS = ["mb_internal.cuh", "mb_ptx.cuh", "mb_decoder.cuh", "mb_gemm.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LINK = ["-Xlinker", "-rpath=/usr/local/cuda/lib64"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build mockbird_b200")


def host_compiler() -> list[str]:
    # nvcc needs a g++ it supports; prefer the system one
    for cand in ("/usr/bin/g++",):
        if os.path.exists(cand):
            return ["-ccbin", cand]
    return []


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "mockbird_kv.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not _stale():
        return LIB
    cmd = [nvcc(), *host_compiler(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC, "-o", LIB + ".tmp",
           *(extra or []), *[os.path.join(CSRC, s) for s in SOURCES], *LINK]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
