"""Runtime gate: torch import, device check, native library load.

Mirrors require_supported_runtime of the reference
(src/tiledattention/_runtime.py:161-191): a module-level lock, a one-shot ready flag,
CUDA availability first, then the compute capability, then the dependencies. The
reference's dependencies are CuPy and cuTile (JIT); here the only dependency is the
ahead-of-time sm_100a library, so the capability gate is narrowed to 10.0 (B200).
"""

from __future__ import annotations

import importlib
from threading import Lock
from types import ModuleType

from ._errors import DependencyError, UnsupportedPlatformError

_SUPPORTED_CC = {(10, 0)}
_runtime_ready = False
_runtime_lock = Lock()
_cached_torch: ModuleType | None = None
_cached_native = None


def _get_torch_module() -> ModuleType:
    global _cached_torch
    if _cached_torch is not None:
        return _cached_torch
    try:
        _cached_torch = importlib.import_module("torch")
        return _cached_torch
    except ModuleNotFoundError as exc:
        raise DependencyError(
            "PyTorch is required for tiledattention. Install a CUDA-enabled torch build first."
        ) from exc


def get_torch_module() -> ModuleType:
    return _get_torch_module()


def _get_native_library():
    """Load the sm_100a shared library (raises DependencyError when absent)."""
    global _cached_native
    if _cached_native is None:
        from . import _native

        _cached_native = _native.load_library()
    return _cached_native


def get_native_library():
    return _get_native_library()


def _query_compute_capability(torch_mod: ModuleType) -> tuple[int, int]:
    try:
        device_index = torch_mod.cuda.current_device()
        major, minor = torch_mod.cuda.get_device_capability(device_index)
        return int(major), int(minor)
    except Exception as exc:  # pragma: no cover - defensive path
        raise UnsupportedPlatformError(
            "Unable to query GPU compute capability from torch.cuda."
        ) from exc


def require_supported_runtime() -> None:
    """Raise UnsupportedPlatformError / DependencyError unless a B200 and the library exist."""
    global _runtime_ready
    if _runtime_ready:  # fast path; the lock below guards the one-time initialisation
        return
    with _runtime_lock:
        if _runtime_ready:
            return
        torch_mod = _get_torch_module()
        if not bool(torch_mod.cuda.is_available()):
            raise UnsupportedPlatformError(
                "tiledattention requires CUDA + Blackwell GPU. "
                "torch.cuda.is_available() is False."
            )
        major, minor = _query_compute_capability(torch_mod)
        if (major, minor) not in _SUPPORTED_CC:
            raise UnsupportedPlatformError(
                f"Unsupported GPU: compute capability {major}.{minor}; "
                "this build targets sm_100a (B200, compute capability 10.0)."
            )
        lib = _get_native_library()
        from . import _native

        fast = _native.load_fast_launch(lib)
        if fast is not None:  # status words created before the launcher was loaded
            from .launch import _status_words

            for idx, word in _status_words.items():
                fast.set_status(idx, word.data_ptr())
        _runtime_ready = True


def _reset_runtime_cache_for_tests() -> None:
    global _runtime_ready, _cached_torch, _cached_native
    with _runtime_lock:
        _runtime_ready = False
        _cached_torch = None
        _cached_native = None
