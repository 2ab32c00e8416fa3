"""The C-ABI library loads and exports every entry point include/*.h declares, and its
argument validation rejects bad calls without touching a GPU. CPU only."""

import ctypes
import glob
import os
import re

import pytest

from tiledattention_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w\s\*]*?\b(ta_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_native.LIB_PATH):
        from tiledattention_b200 import build

        build.build()
    return _native.load_library(_native.LIB_PATH)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ta_sdpa_fwd" in names and len(names) >= 5


def test_every_declared_symbol_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} missing from the ctypes binding"


def test_abi_version_and_strings(lib):
    assert lib.ta_abi_version() >= 100
    assert _native.status_string(lib, 0) == "ok"
    assert "head dim" in _native.status_string(lib, _native.TA_ERR_UNSUPPORTED_DIM)


def _call(lib, D=128, dtype=1, scale=0.1, null_q=False, S=64, ostride3=1):
    st = _native.strides4([2 * S * D, S * D, D, 1])
    ost = _native.strides4([2 * S * D, S * D, D, ostride3])
    p = None if null_q else 0x1000
    return lib.ta_sdpa_fwd(p, 0x1000, 0x1000, 0x1000, None, 1, 2, S, D, st, st, st, ost,
                           dtype, 1, scale, None, None)


def test_argument_validation_without_gpu(lib):
    assert _call(lib, null_q=True) == _native.TA_ERR_INVALID_ARGUMENT
    # native 64/128/256, or another multiple of 8 up to 256 (run without padding); others
    # rejected
    assert _call(lib, D=100) == _native.TA_ERR_UNSUPPORTED_DIM
    assert _call(lib, D=264) == _native.TA_ERR_UNSUPPORTED_DIM
    assert _call(lib, D=4) == _native.TA_ERR_UNSUPPORTED_DIM
    assert _call(lib, dtype=7) == _native.TA_ERR_UNSUPPORTED_DTYPE
    assert _call(lib, scale=0.0) == _native.TA_ERR_INVALID_ARGUMENT
    assert _call(lib, scale=float("inf")) == _native.TA_ERR_INVALID_ARGUMENT
    assert _call(lib, S=0) == _native.TA_ERR_INVALID_ARGUMENT
    assert _call(lib, ostride3=2) == _native.TA_ERR_LAYOUT
    assert "stride" in _native.last_error(lib)


def test_devstat_description():
    assert "softmax" in _native.describe_devstat(4)
    assert "MMA" in _native.describe_devstat(2)


def test_merge_head_dims_without_gpu(lib):
    # The split-KV merges take any multiple of 8 up to 256 (the state of an unpadded head
    # dim); other head dims are rejected before any device work.
    st = _native.strides4([2 * 64 * 100, 64 * 100, 100, 1])
    for D in (100, 4, 264):
        rc = lib.ta_lse_combine(0x1000, 0x1000, 2, 1, 2, 64, D, 0x1000, st, 1, None, None)
        assert rc == _native.TA_ERR_UNSUPPORTED_DIM, D
    ptrs = (ctypes.c_void_p * 1)(0x1000)
    fptrs = (ctypes.POINTER(ctypes.c_float) * 1)()
    for D in (100, 4, 264):
        rc = lib.ta_lse_merge_peers(ptrs, ptrs, 1, 1, 2, 64, D, 0, 64, ptrs, fptrs, 1, st, 64, 0,
                                    1, None, None)
        assert rc == _native.TA_ERR_UNSUPPORTED_DIM, D


def test_noalloc_head_dims_without_gpu(lib):
    st = _native.strides4([2 * 64 * 100, 64 * 100, 100, 1])
    for D in (100, 4, 264):
        rc = lib.ta_sdpa_fwd_split_noalloc(16, 16, 16, 16, None, 1, 2, 64, D, st, st, st, st,
                                           _native.TA_DTYPE_BF16, 1, 0.1, 2, None, None)
        assert rc == _native.TA_ERR_UNSUPPORTED_DIM, D
