"""Ahead-of-time build of the sm_100a native library (replaces the reference's
cuTile JIT + compile cache, src/tiledattention/kernels/compile_cache.py:10-37).

    python -m tiledattention_b200.build

compiles csrc/*.cu with nvcc for sm_100a into _lib/libtiledattention_b200.so
(in-tree, so the built library travels with the source tree). Every variant
(kernel head dim 64/128/256 x fp16/bf16 x causal/non-causal x 16-bit/fp32-partial output)
is instantiated at build time; any head dim that is a multiple of 8 up to 256 runs on the
next kernel head dim without padded copies.
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
SOURCES = ["capi.cu", "sdpa_fwd_sm100.cu", "sdpa_fwd_sm100_shared_kv.cu", "lse_combine.cu", "noalloc_split.cu", "peer_merge.cu"]
HEADERS = ["sm100_ptx.cuh", "sdpa_common.cuh", "sdpa_fwd_sm100.h", "lse_combine.h", "capi_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# One-call host launcher (CPython extension over libtorch; no device code): see
# csrc/fast_launch.cpp.
FAST_SOURCE = "fast_launch.cpp"


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


def fast_launch_path() -> str:
    import sysconfig

    return os.path.join(OUT_DIR, "_fast_launch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fast_launch(force: bool = False) -> str:
    """Compile csrc/fast_launch.cpp with the host C++ compiler against the installed torch."""
    import sysconfig

    import torch

    out = fast_launch_path()
    src = os.path.join(CSRC, FAST_SOURCE)
    deps = (src, os.path.join(REPO_DIR, "include", "tiledattention_b200.h"))
    stamp = out + ".torch"  # the torch version the module was built against (C++ ABI)
    built_for = open(stamp).read().strip() if os.path.exists(stamp) else None
    if not force and os.path.exists(out) and built_for == torch.__version__ and all(
            os.path.getmtime(out) >= os.path.getmtime(d) for d in deps):
        return out
    torch_dir = os.path.dirname(torch.__file__)
    cuda_home = os.environ.get("CUDA_HOME") or os.path.dirname(os.path.dirname(nvcc_path()))
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-I", os.path.join(torch_dir, "include"),
        "-I", os.path.join(torch_dir, "include", "torch", "csrc", "api", "include"),
        "-I", os.path.join(cuda_home, "include"),
        "-I", sysconfig.get_paths()["include"],
        "-I", os.path.join(REPO_DIR, "include"),
        src, "-o", out + ".tmp",
        "-L", os.path.join(torch_dir, "lib"), "-lc10", "-lc10_cuda", "-ltorch_cpu",
        "-ltorch_python", "-Wl,-rpath," + os.path.join(torch_dir, "lib"),
    ]
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    with open(stamp, "w") as f:
        f.write(torch.__version__ + "\n")
    return out


def build(force: bool = False, verbose: bool = False) -> str:
    build_fast_launch(force)
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
