"""ctypes binding of the C ABI declared in include/tiledattention_b200.h.

The shared library is built ahead of time for sm_100a (tiledattention_b200/build.py)
and lives in-tree at tiledattention_b200/_lib/libtiledattention_b200.so. There is no
fallback: if the library is missing, loading raises DependencyError.
"""

from __future__ import annotations

import ctypes
import os
import threading

from ._errors import DependencyError

LIB_NAME = "libtiledattention_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", LIB_NAME)

# Status codes (include/tiledattention_b200.h).
TA_OK = 0
TA_ERR_INVALID_ARGUMENT = 1
TA_ERR_UNSUPPORTED_DIM = 2
TA_ERR_UNSUPPORTED_DTYPE = 3
TA_ERR_LAYOUT = 4
TA_ERR_CUDA = 5
TA_ERR_DRIVER = 6
TA_ERR_DEVICE = 7

TA_DTYPE_F16 = 0
TA_DTYPE_BF16 = 1
TA_MAX_PEERS = 8
TA_DTYPE_F32 = 2

DEVSTAT_BITS = {
    1: "TMA producer wait timed out",
    2: "MMA issuer wait timed out",
    4: "softmax wait timed out",
    8: "epilogue wait timed out",
    16: "drain of in-flight copies/MMAs timed out",
    32: "peer barrier timed out (a peer GPU did not arrive)",
}

# Every symbol include/tiledattention_b200.h declares, with its ctypes signature.
_I64P = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    # stride arguments as plain addresses (ctypes arrays or ints), for a cheap hot call
    "ta_sdpa_fwd": (
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
        ],
    ),
    "ta_sdpa_fwd_partial": (
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            _I64P, _I64P, _I64P,
            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p,
        ],
    ),
    "ta_lse_combine": (
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, _I64P, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ],
    ),
    "ta_peer_barrier": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint, ctypes.c_ulonglong,
         ctypes.c_void_p, ctypes.c_void_p],
    ),
    "ta_lse_merge_peers": (
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, _I64P, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ],
    ),
    "ta_sdpa_fwd_split_noalloc": (
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            _I64P, _I64P, _I64P, _I64P,
            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p,
        ],
    ),
    "ta_device_supported": (ctypes.c_int, [ctypes.c_int]),
    "ta_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ta_last_error": (ctypes.c_char_p, []),
    "ta_abi_version": (ctypes.c_int, []),
    "ta_debug_set_selftest": (None, [ctypes.c_int, ctypes.c_ulonglong]),
    "ta_debug_set_kernel": (None, [ctypes.c_int]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library with its signatures applied."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        # TILEDATTN_NATIVE_LIB: load another build of the same ABI (A/B experiments).
        lib_path = path or os.environ.get("TILEDATTN_NATIVE_LIB") or LIB_PATH
        if not os.path.exists(lib_path):
            raise DependencyError(
                f"native library {lib_path} not found; build it with "
                "`python -m tiledattention_b200.build`."
            )
        try:
            lib = ctypes.CDLL(lib_path)
        except OSError as exc:
            raise DependencyError(f"cannot load {lib_path}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def last_error(lib: ctypes.CDLL) -> str:
    msg = lib.ta_last_error()
    return msg.decode() if msg else ""


def status_string(lib: ctypes.CDLL, code: int) -> str:
    msg = lib.ta_status_string(code)
    return msg.decode() if msg else ""


def strides4(strides) -> ctypes.Array:
    arr = (ctypes.c_int64 * 4)(*[int(s) for s in strides])
    return arr


_I64x16 = ctypes.c_int64 * 16
_I64_SIZE = ctypes.sizeof(ctypes.c_int64)


def strides16(*stride_tuples):
    """Four 4-element stride tuples packed in one ctypes array; returns the addresses of
    its four sub-arrays and the array itself (keep the tuple alive during the call)."""
    arr = _I64x16(*[int(x) for t in stride_tuples for x in t])
    base = ctypes.addressof(arr)
    return (base, base + 4 * _I64_SIZE, base + 8 * _I64_SIZE, base + 12 * _I64_SIZE, arr)


def describe_devstat(word: int) -> str:
    parts = [text for bit, text in DEVSTAT_BITS.items() if word & bit]
    return "; ".join(parts) if parts else f"status 0x{word:x}"


_fast = None
_fast_tried = False


def load_fast_launch(lib):
    """Load (once) the one-call host launcher (_lib/_fast_launch*.so, built from
    csrc/fast_launch.cpp) and bind it to `lib`'s entry points. Loading it also registers the
    C++ torch operators torch.ops.tiledattention_b200.sdpa_fwd / sdpa_fwd_partial. Returns
    the module, or None when it is not built or disabled (the Python launch path then takes
    every call and tiledattention_b200.ops registers the operators in Python)."""
    global _fast, _fast_tried
    if not isinstance(lib, ctypes.CDLL):
        return None
    with _lock:
        if _fast_tried:
            return _fast
        _fast_tried = True
        if os.environ.get("TILEDATTN_FAST_LAUNCH", "1") == "0":
            return None
        import importlib.util
        import sysconfig

        path = os.path.join(os.path.dirname(LIB_PATH),
                            "_fast_launch" + sysconfig.get_config_var("EXT_SUFFIX"))
        if not os.path.exists(path):  # not built for this interpreter
            return None
        import torch

        stamp = path + ".torch"
        if not os.path.exists(stamp) or open(stamp).read().strip() != torch.__version__:
            return None  # built against another torch: its C++ ABI may differ
        spec = importlib.util.spec_from_file_location("tiledattention_b200._fast_launch", path)
        mod = importlib.util.module_from_spec(spec)
        try:
            spec.loader.exec_module(mod)
        except ImportError:  # built against another torch: the Python launch path remains
            return None
        addr = lambda fn: ctypes.cast(fn, ctypes.c_void_p).value  # noqa: E731
        mod.set_entry(addr(lib.ta_sdpa_fwd))
        mod.bind_ops(addr(lib.ta_sdpa_fwd_partial), addr(lib.ta_last_error))
        _fast = mod
        return mod


def fast_launch_module():
    """The loaded one-call launcher module, or None."""
    return _fast
