"""torch operator registration: the native-op slot of the reference's kernel-builder build.

The reference registers its CUDA ops in ``torch-ext/torch_binding.cpp:6-19`` (a stub there).
Importing this module makes these operators available:

    torch.ops.tiledattention_b200.sdpa_fwd(q, k, v, causal, scale) -> Tensor
    torch.ops.tiledattention_b200.sdpa_fwd_partial(q, k, v, causal, scale, kv_begin, kv_end,
                                                   n_split) -> (Tensor o_f32, Tensor lse_f32)

``scale`` is explicit (the Python API's ``scale=None`` default, 1/sqrt(D), is resolved by
``tiledattention_b200.sdpa``). Normally they are the C++ operators of
``csrc/fast_launch.cpp`` (registered with TORCH_LIBRARY when the package's native launcher
module loads: CUDA kernels over the C ABI, Meta kernels for shapes, errors raised with
TORCH_CHECK as the reference's stub does). Where that module is not built or is disabled
(``TILEDATTN_FAST_LAUNCH=0``) they are registered here with ``torch.library.custom_op`` over
the Python launch path, with fake implementations, raising the package's errors. Either way
the ops run the sm_100a kernels on the current stream and trace under ``torch.compile``.
"""

from __future__ import annotations

import torch

from . import _native
from ._errors import DependencyError
from .launch import run_sdpa_partial
from .sdpa import _prepare, sdpa as _sdpa

_NS = "tiledattention_b200"


def _native_ops_module():
    """The loaded native launcher module (whose loading registered the C++ operators), or
    None."""
    try:
        lib = _native.load_library()
    except DependencyError:
        return None
    return _native.load_fast_launch(lib)


NATIVE_OPS = _native_ops_module() is not None


if NATIVE_OPS:
    sdpa_fwd = torch.ops.tiledattention_b200.sdpa_fwd
    sdpa_fwd_partial = torch.ops.tiledattention_b200.sdpa_fwd_partial
else:
    @torch.library.custom_op(f"{_NS}::sdpa_fwd", mutates_args=())
    def sdpa_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                 scale: float) -> torch.Tensor:
        """softmax(q k^T * scale + causal mask) v over [B,H,S,D] fp16/bf16 CUDA tensors."""
        return _sdpa(q, k, v, causal=causal, scale=scale)

    @sdpa_fwd.register_fake
    def _sdpa_fwd_fake(q, k, v, causal, scale):
        return torch.empty(q.shape, dtype=q.dtype, device=q.device)

    @torch.library.custom_op(f"{_NS}::sdpa_fwd_partial", mutates_args=())
    def sdpa_fwd_partial(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                         scale: float, kv_begin: int, kv_end: int,
                         n_split: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Split-KV partials over keys [kv_begin, kv_end) cut into n_split slices:
        fp32 o [n_split,B,H,S,D] (each slice normalised by its own row sum) and fp32 natural-log
        lse [n_split,B,H,S] (-inf where a slice has no valid key for the row)."""
        resolved = _prepare(q, k, v, causal, scale)
        o, lse = run_sdpa_partial(q, k, v, causal=causal, scale=resolved, kv_begin=kv_begin,
                                  kv_end=kv_end, n_split=n_split)
        head_dim = int(q.shape[-1])
        if o.shape[-1] != head_dim:
            o = o[..., :head_dim].contiguous()
        return o, lse

    @sdpa_fwd_partial.register_fake
    def _sdpa_fwd_partial_fake(q, k, v, causal, scale, kv_begin, kv_end, n_split):
        b, h, s, d = q.shape
        o = torch.empty((n_split, b, h, s, d), dtype=torch.float32, device=q.device)
        lse = torch.empty((n_split, b, h, s), dtype=torch.float32, device=q.device)
        return o, lse
