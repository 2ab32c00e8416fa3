"""tiledattention_b200 — B200-native (sm_100a) scaled-dot-product-attention forward.

Drop-in for the public API of thisistaimur/TiledAttention
(src/tiledattention/__init__.py:20-55): ``sdpa(q, k, v, *, causal=False, scale=None)``
and the exception classes. The ``sdpa`` submodule is imported eagerly and the
function re-bound afterwards, so ``tiledattention_b200.sdpa`` stays the function
(the reference's lazy import replaces it by the submodule after the first call).
"""

from __future__ import annotations

from . import sdpa as _sdpa_module  # noqa: F401  (binds the submodule before the function)
from ._errors import (
    DependencyError,
    DTypeNotSupportedError,
    InvalidShapeError,
    KernelError,
    TiledAttentionError,
    UnsupportedPlatformError,
)
from ._version import __version__
from .launch import check_device_status
from .sdpa import sdpa, sdpa_partial, sdpa_split_kv, sdpa_with_lse

__all__ = [
    "__version__",
    "sdpa",
    "sdpa_with_lse",
    "sdpa_split_kv",
    "sdpa_partial",
    "check_device_status",
    "TiledAttentionError",
    "UnsupportedPlatformError",
    "InvalidShapeError",
    "DTypeNotSupportedError",
    "DependencyError",
    "KernelError",
]
