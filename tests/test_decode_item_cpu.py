"""The persistent kernels' work-item decode (csrc/sdpa_common.cuh, decode_item), compiled by
nvcc for the host and run on the CPU over a sweep of shapes, group sizes, key ranges and
slice counts: every (slice, (b,h) pair, query block) exactly once, in slice / group order
with the longest causal blocks of a group first, and the key ranges the masks imply."""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_decode_item_order_and_coverage(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    exe = str(tmp_path / "decode_item_check")
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "native", "decode_item_check.cu"), "-o", exe],
                   check=True, capture_output=True, timeout=600)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok "), r.stdout
    assert int(r.stdout.split()[1]) > 1000
