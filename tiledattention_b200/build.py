"""Ahead-of-time build of the sm_100a native library (replaces the reference's
cuTile JIT + compile cache, src/tiledattention/kernels/compile_cache.py:10-37).

    python -m tiledattention_b200.build

compiles csrc/*.cu with nvcc for sm_100a into _lib/libtiledattention_b200.so
(in-tree, so the built library travels with the source tree). Every variant
(head dim 64/128 x fp16/bf16 x causal/non-causal) is instantiated at build time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
OUT_DIR = os.path.join(PKG_DIR, "_lib")
OUT = os.path.join(OUT_DIR, "libtiledattention_b200.so")
SOURCES = ["capi.cu", "sdpa_fwd_sm100.cu", "sdpa_fwd_sm100_shared_kv.cu", "sdpa_fwd_sm100_pair.cu", "lse_combine.cu", "noalloc_split.cu", "peer_merge.cu"]
HEADERS = ["sm100_ptx.cuh", "sm100_pair.cuh", "sdpa_common.cuh", "sdpa_fwd_sm100.h", "lse_combine.h", "capi_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO_DIR, "include", "tiledattention_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [
        nvcc_path(), "-O3", "-std=c++17", *ARCH, "-lineinfo",
        "-Xcompiler", "-fPIC", "-shared",
        "-I", os.path.join(REPO_DIR, "include"),
        "-o", OUT + ".tmp",
        *[os.path.join(CSRC, f) for f in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
