"""PyTorch-facing SDPA API.

sdpa(q, k, v, *, causal=False, scale=None) -> o, the drop-in for the reference's
src/tiledattention/sdpa.py:14-48: scalar checks first (non-bool causal or
non-positive scale -> InvalidShapeError), then the runtime gate, then the tensor
contract, then scale = 1/sqrt(D) of the original head dim, then the launch.
"""

from __future__ import annotations

import math
import os
from numbers import Real

from . import _native, _runtime
from ._errors import InvalidShapeError
from .checks import validate_sdpa_inputs
from .launch import run_lse_combine, run_sdpa_fwd, run_sdpa_partial


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


def _fast_launch(q, k, v, causal, scale, want_lse):
    """The one-call native launcher for the common case, or None (the full path then runs
    and raises the reference's error, copies or pads as needed). Taken only once the runtime
    gate has passed and with the default asynchronous sync mode."""
    fast = _native._fast
    if fast is None or not _runtime._runtime_ready:
        return None
    mode = os.environ.get("TILEDATTN_SYNC_MODE")
    if mode is not None and mode.strip().lower() != "async":
        return None
    if scale is None:
        scale = -1.0  # the launcher's code for 1/sqrt(D)
    elif scale.__class__ is not float or not scale > 0:
        return None
    return fast.launch(q, k, v, causal, scale, want_lse)


def sdpa(q, k, v, *, causal: bool = False, scale: float | None = None):
    """Scaled dot-product attention forward: softmax(q k^T * scale + mask) v.

    q, k, v: [B, H, S, D] CUDA tensors, float16 or bfloat16, identical shape/dtype/device.
    causal:  top-left causal mask (query row i attends to keys 0..i).
    scale:   positive float; defaults to 1/sqrt(D).
    Returns a new [B, H, S, D] tensor of q's dtype, computed asynchronously on the
    current torch stream.
    """
    out = _fast_launch(q, k, v, causal, scale, False)
    if out is not None:
        return out
    resolved_scale = _prepare(q, k, v, causal, scale)
    return run_sdpa_fwd(q, k, v, causal=causal, scale=resolved_scale)


def sdpa_with_lse(q, k, v, *, causal: bool = False, scale: float | None = None):
    """Like sdpa, and also returns the float32 [B, H, S] log-sum-exp of the scaled scores.

    The reference has no lse output; it is the building block of the split-KV merge.
    """
    out = _fast_launch(q, k, v, causal, scale, True)
    if out is not None:
        return out
    resolved_scale = _prepare(q, k, v, causal, scale)
    return run_sdpa_fwd(q, k, v, causal=causal, scale=resolved_scale, return_lse=True)


def sdpa_split_kv(q, k, v, *, causal: bool = False, scale: float | None = None,
                  n_split: int = 4, return_lse: bool = False):
    """sdpa computed as n_split key slices in one launch plus a log-sum-exp merge.

    Same result as sdpa (up to fp32 rounding); useful when B*H*ceil(S/256) is small
    compared with the 148 SMs of a B200 (long sequences with few heads, decode-like
    shapes). The reference has no split-KV mode.
    """
    resolved_scale = _prepare(q, k, v, causal, scale)
    if not isinstance(n_split, int) or n_split < 1:
        raise InvalidShapeError("n_split must be a positive int.")
    o_part, lse_part = run_sdpa_partial(q, k, v, causal=causal, scale=resolved_scale,
                                        n_split=n_split)
    return run_lse_combine(o_part, lse_part, out_dtype=q.dtype, head_dim=int(q.shape[-1]),
                           return_lse=return_lse)


def sdpa_partial(q, k, v, *, causal: bool = False, scale: float | None = None,
                 kv_begin: int = 0, kv_end: int | None = None, n_split: int = 1):
    """Attention of all query rows over the keys [kv_begin, kv_end) only (split into
    n_split slices): returns fp32 (o_part [n_split,B,H,S,D], lse_part [n_split,B,H,S])."""
    resolved_scale = _prepare(q, k, v, causal, scale)
    o_part, lse_part = run_sdpa_partial(q, k, v, causal=causal, scale=resolved_scale,
                                        kv_begin=kv_begin, kv_end=kv_end, n_split=n_split)
    head_dim = int(q.shape[-1])
    return (o_part[..., :head_dim] if o_part.shape[-1] != head_dim else o_part), lse_part
