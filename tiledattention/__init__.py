"""Drop-in import name: ``import tiledattention`` resolves to tiledattention_b200.

Code written against thisistaimur/TiledAttention (``tiledattention.sdpa(...)``,
``from tiledattention.sdpa import sdpa``, the exception classes) runs unchanged.
"""

from __future__ import annotations

from tiledattention_b200 import (  # noqa: F401
    DependencyError,
    DTypeNotSupportedError,
    InvalidShapeError,
    KernelError,
    TiledAttentionError,
    UnsupportedPlatformError,
    __version__,
    check_device_status,
    sdpa_partial,
    sdpa_split_kv,
    sdpa_with_lse,
)

from . import sdpa as _sdpa_module  # noqa: F401,E402
from .sdpa import sdpa  # noqa: E402

__all__ = [
    "__version__",
    "sdpa",
    "TiledAttentionError",
    "UnsupportedPlatformError",
    "InvalidShapeError",
    "DTypeNotSupportedError",
    "DependencyError",
]
