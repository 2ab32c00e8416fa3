"""Exception hierarchy of the SDPA operator.

Same class names and meaning as the reference package
(src/tiledattention/_errors.py:6-23 of thisistaimur/TiledAttention), so callers that
catch them keep working after switching to this package.
"""

from __future__ import annotations


class TiledAttentionError(Exception):
    """Base exception for tiledattention."""


class UnsupportedPlatformError(TiledAttentionError):
    """Raised when runtime platform requirements are not satisfied."""


class InvalidShapeError(TiledAttentionError):
    """Raised when q/k/v tensors do not match expected SDPA input contracts."""


class DTypeNotSupportedError(TiledAttentionError):
    """Raised when input tensor dtypes are unsupported."""


class DependencyError(TiledAttentionError):
    """Raised when a required dependency is missing."""


class KernelError(TiledAttentionError):
    """Raised when the native kernel reports a failure (launch error or device status)."""
