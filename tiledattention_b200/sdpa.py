"""PyTorch-facing SDPA API.

sdpa(q, k, v, *, causal=False, scale=None) -> o, the drop-in for the reference's
src/tiledattention/sdpa.py:14-48: scalar checks first (non-bool causal or
non-positive scale -> InvalidShapeError), then the runtime gate, then the tensor
contract, then scale = 1/sqrt(D) of the original head dim, then the launch.
"""

from __future__ import annotations

import math
from numbers import Real

from . import _runtime
from ._errors import InvalidShapeError
from .checks import validate_sdpa_inputs
from .launch import run_sdpa_fwd


def _prepare(q, k, v, causal, scale):
    if not isinstance(causal, bool):
        raise InvalidShapeError("causal must be a bool.")
    if scale is not None and (not isinstance(scale, Real) or not float(scale) > 0):
        raise InvalidShapeError("scale must be a positive number when provided.")
    _runtime.require_supported_runtime()
    torch_mod = _runtime.get_torch_module()
    validate_sdpa_inputs(torch_mod, q, k, v)
    head_dim = int(q.shape[-1])
    return float(scale) if scale is not None else 1.0 / math.sqrt(head_dim)


def sdpa(q, k, v, *, causal: bool = False, scale: float | None = None):
    """Scaled dot-product attention forward: softmax(q k^T * scale + mask) v.

    q, k, v: [B, H, S, D] CUDA tensors, float16 or bfloat16, identical shape/dtype/device.
    causal:  top-left causal mask (query row i attends to keys 0..i).
    scale:   positive float; defaults to 1/sqrt(D).
    Returns a new [B, H, S, D] tensor of q's dtype, computed asynchronously on the
    current torch stream.
    """
    resolved_scale = _prepare(q, k, v, causal, scale)
    return run_sdpa_fwd(q, k, v, causal=causal, scale=resolved_scale)


def sdpa_with_lse(q, k, v, *, causal: bool = False, scale: float | None = None):
    """Like sdpa, and also returns the float32 [B, H, S] log-sum-exp of the scaled scores.

    The reference has no lse output; it is the building block of the split-KV merge.
    """
    resolved_scale = _prepare(q, k, v, causal, scale)
    return run_sdpa_fwd(q, k, v, causal=causal, scale=resolved_scale, return_lse=True)
