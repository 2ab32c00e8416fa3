"""Host launcher: layout policy, output allocation and the call through the C ABI.

Replaces run_flash_fwd (src/tiledattention/kernels/flash_fwd.py:821-973) and
_launch_cutile_kernel (flash_fwd.py:786-818) of the reference:
  * no reshape / transpose copies: each operand keeps its own strides, which the C
    ABI turns into TMA tensor maps; only layouts TMA cannot express (head-dim stride
    != 1, strides or base not 16-byte aligned) are made contiguous first, as the
    reference does unconditionally (flash_fwd.py:865-867);
  * head dims other than 64/128/256 are zero-padded to the next supported size
    (flash_fwd.py:149-163, 868-872); the scale is resolved by the caller from the
    original head dim (sdpa.py:46-47), so padding does not change the result;
  * the output is a fresh tensor like empty_like(q) (flash_fwd.py:877);
  * the launch goes on torch's current stream of q's device (the reference launches
    on CuPy's current stream, flash_fwd.py:805-809);
  * TILEDATTN_SYNC_MODE = async (default) | post | strict keeps the reference's debug
    sync semantics (flash_fwd.py:805-818); post/strict also read the kernel's device
    status word and raise KernelError if a bounded wait in the kernel expired.
"""

from __future__ import annotations

import contextlib
import os

from . import _native, _runtime
from ._errors import (
    DTypeNotSupportedError,
    InvalidShapeError,
    KernelError,
    UnsupportedPlatformError,
)

NATIVE_HEAD_DIMS = (64, 128, 256)
_NULL_CTX = contextlib.nullcontext()


def _raw_stream(torch_mod, dev_idx: int) -> int:
    """cudaStream_t of torch's current stream on device dev_idx (fast path when available)."""
    raw = getattr(torch_mod._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(dev_idx)
    return torch_mod.cuda.current_stream(dev_idx).cuda_stream
_status_words: dict[int, object] = {}


def padded_head_dim(head_dim: int) -> int:
    """Head dim the kernel runs at for a given input head dim."""
    for d in NATIVE_HEAD_DIMS:
        if head_dim <= d:
            return d
    raise InvalidShapeError(
        f"head dim {head_dim} is not supported (this build supports head dims up to 256)."
    )


def state_head_dim(head_dim: int) -> int:
    """Head dim of the split-KV state (partials, merged outputs) for an input head dim: the
    head dim itself when it is a multiple of 8 (the kernels read and write it without
    padding), else the padded native size."""
    if head_dim % 8 == 0 and 0 < head_dim <= NATIVE_HEAD_DIMS[-1]:
        return head_dim
    return padded_head_dim(head_dim)


def _status_word(torch_mod, device):
    idx = device.index if device.index is not None else torch_mod.cuda.current_device()
    word = _status_words.get(idx)
    if word is None:
        word = torch_mod.zeros(1, dtype=torch_mod.int32, device=device)
        _status_words[idx] = word
        fast = _native.fast_launch_module()
        if fast is not None:
            fast.set_status(idx, word.data_ptr())
    return word


def check_device_status(device=None) -> None:
    """Synchronise `device` and raise KernelError if a kernel reported a timeout."""
    torch_mod = _runtime.get_torch_module()
    if device is None:
        device = torch_mod.device("cuda", torch_mod.cuda.current_device())
    word = _status_word(torch_mod, torch_mod.device(device))
    torch_mod.cuda.synchronize(word.device)
    value = int(word.item())
    if value:
        word.zero_()
        raise KernelError("tiledattention kernel: " + _native.describe_devstat(value))


def _tma_compatible(t) -> bool:
    if t.is_contiguous():  # [B,H,S,D] contiguous: strides are multiples of D (16-bit, D >= 64)
        return t.data_ptr() % 16 == 0
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        return False
    for dim in range(3):
        if t.size(dim) > 1 and (t.stride(dim) * t.element_size()) % 16:
            return False
    return True


def _sync_mode() -> str:
    """TILEDATTN_SYNC_MODE, as the reference reads it (flash_fwd.py:805-818): an unknown
    value raises the reference's ValueError instead of silently running asynchronously."""
    mode = os.getenv("TILEDATTN_SYNC_MODE", "async").strip().lower()
    if mode not in ("async", "post", "strict"):
        raise ValueError(
            f"Unsupported TILEDATTN_SYNC_MODE={mode!r}. Use one of: strict, post, async.")
    return mode


def run_sdpa_fwd(q, k, v, *, causal: bool, scale: float, return_lse: bool = False):
    """Launch the sm_100a kernel. Inputs are already validated ([B,H,S,D], fp16/bf16, CUDA).

    Returns o (and the float32 [B,H,S] natural-log log-sum-exp when return_lse=True).
    Head dims 64/128/256 run natively; another multiple of 8 runs without padded copies
    (the kernel zero-fills the missing columns on load and writes only the true columns);
    other head dims are zero-padded to the next native size.
    """
    torch_mod = _runtime.get_torch_module()
    lib = _runtime.get_native_library()
    batch, heads, seq_len, head_dim = (int(x) for x in q.shape)
    kdim = padded_head_dim(head_dim)
    if q.dtype == torch_mod.float16:
        dtype_code = _native.TA_DTYPE_F16
    elif q.dtype == torch_mod.bfloat16:
        dtype_code = _native.TA_DTYPE_BF16
    else:  # validated earlier; kept for direct callers
        raise DTypeNotSupportedError("q dtype must be torch.float16 or torch.bfloat16.")

    lse = None
    if return_lse:
        lse = torch_mod.empty((batch, heads, seq_len), dtype=torch_mod.float32, device=q.device)
    if q.numel() == 0:
        out = torch_mod.empty((batch, heads, seq_len, head_dim), dtype=q.dtype, device=q.device)
        return (out, lse) if return_lse else out

    mode = _sync_mode()
    dev_idx = q.device.index if q.device.index is not None else torch_mod.cuda.current_device()
    switch = dev_idx != torch_mod.cuda.current_device()
    ctx = torch_mod.cuda.device(dev_idx) if switch else _NULL_CTX
    with ctx:
        status = _status_word(torch_mod, q.device)
        stream = _raw_stream(torch_mod, dev_idx)
        if mode == "strict":
            torch_mod.cuda.synchronize(q.device)

        def launch(qq, kk, vv, out, dim):
            st = _native.strides16(qq.stride(), kk.stride(), vv.stride(), out.stride())
            return lib.ta_sdpa_fwd(
                qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), out.data_ptr(),
                lse.data_ptr() if lse is not None else None,
                batch, heads, seq_len, dim, st[0], st[1], st[2], st[3],
                dtype_code, 1 if causal else 0, float(scale), status.data_ptr(), stream,
            )

        rc = _native.TA_ERR_UNSUPPORTED_DIM
        if kdim == head_dim or head_dim % 8 == 0:
            out = torch_mod.empty((batch, heads, seq_len, head_dim), dtype=q.dtype,
                                  device=q.device)
            qa, ka, va = (t if _tma_compatible(t) else t.contiguous() for t in (q, k, v))
            rc = launch(qa, ka, va, out, head_dim)
            if rc == _native.TA_ERR_LAYOUT and not all(t.is_contiguous() for t in (qa, ka, va)):
                qa, ka, va = qa.contiguous(), ka.contiguous(), va.contiguous()
                rc = launch(qa, ka, va, out, head_dim)
        if rc == _native.TA_ERR_UNSUPPORTED_DIM and kdim != head_dim:
            # Zero-pad to the next native head dim (flash_fwd.py:868-872 pads the same way).
            pad = (0, kdim - head_dim)
            qp, kp, vp = (torch_mod.nn.functional.pad(t, pad) for t in (q, k, v))
            full = torch_mod.empty((batch, heads, seq_len, kdim), dtype=q.dtype, device=q.device)
            rc = launch(qp, kp, vp, full, kdim)
            out = full[..., :head_dim]
        if rc != _native.TA_OK:
            _raise_for(lib, rc)
        if mode in ("post", "strict"):
            check_device_status(q.device)

    return (out, lse) if return_lse else out


def _dtype_code(torch_mod, dtype):
    if dtype == torch_mod.float16:
        return _native.TA_DTYPE_F16
    if dtype == torch_mod.bfloat16:
        return _native.TA_DTYPE_BF16
    raise DTypeNotSupportedError("q dtype must be torch.float16 or torch.bfloat16.")


def _raise_for(lib, rc):
    detail = _native.last_error(lib) or _native.status_string(lib, rc)
    if rc == _native.TA_ERR_DEVICE:
        raise UnsupportedPlatformError(detail)
    if rc in (_native.TA_ERR_INVALID_ARGUMENT, _native.TA_ERR_UNSUPPORTED_DIM, _native.TA_ERR_LAYOUT):
        raise InvalidShapeError(detail)
    if rc == _native.TA_ERR_UNSUPPORTED_DTYPE:
        raise DTypeNotSupportedError(detail)
    raise KernelError(detail)


def run_sdpa_partial(q, k, v, *, causal: bool, scale: float, kv_begin: int = 0,
                     kv_end: int | None = None, n_split: int = 1, out=None):
    """Split-KV forward over keys [kv_begin, kv_end) cut into n_split slices.

    Returns (o_part, lse_part): fp32 [n_split, B, H, S, Dk] (each slice normalised by its
    own row sum) and fp32 [n_split, B, H, S] natural-log log-sum-exp (-inf where a slice
    has no valid key for the row). Dk = state_head_dim(D): D itself for multiples of 8,
    else the padded native size, whose extra columns the caller slices off. Inputs are already validated. ``out`` = (o_part,
    lse_part): contiguous fp32 tensors of those shapes to write into (e.g. views of a
    buffer the peers have mapped) instead of new ones.
    """
    torch_mod = _runtime.get_torch_module()
    lib = _runtime.get_native_library()
    batch, heads, seq_len, head_dim = (int(x) for x in q.shape)
    kdim = state_head_dim(head_dim)
    kv_end = seq_len if kv_end is None else int(kv_end)
    dtype_code = _dtype_code(torch_mod, q.dtype)
    if out is not None:
        o_part, lse_part = out
        if (tuple(o_part.shape) != (n_split, batch, heads, seq_len, kdim)
                or tuple(lse_part.shape) != (n_split, batch, heads, seq_len)
                or o_part.dtype != torch_mod.float32 or lse_part.dtype != torch_mod.float32
                or not o_part.is_contiguous() or not lse_part.is_contiguous()
                or o_part.data_ptr() % 16):
            raise InvalidShapeError("out: contiguous fp32 [n_split,B,H,S,Dk] and [n_split,B,H,S] "
                                    "tensors (16-byte aligned) required")
    else:
        o_part = torch_mod.empty((n_split, batch, heads, seq_len, kdim), dtype=torch_mod.float32,
                                 device=q.device)
        lse_part = torch_mod.empty((n_split, batch, heads, seq_len), dtype=torch_mod.float32,
                                   device=q.device)
    if o_part.numel() == 0:
        return o_part, lse_part
    if kdim != head_dim:
        pad = (0, kdim - head_dim)
        q, k, v = (torch_mod.nn.functional.pad(t, pad) for t in (q, k, v))
    q, k, v = (t if _tma_compatible(t) else t.contiguous() for t in (q, k, v))
    with torch_mod.cuda.device(q.device):
        status = _status_word(torch_mod, q.device)
        stream = torch_mod.cuda.current_stream(q.device).cuda_stream
        rc = lib.ta_sdpa_fwd_partial(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o_part.data_ptr(), lse_part.data_ptr(),
            batch, heads, seq_len, kdim,
            _native.strides4(q.stride()), _native.strides4(k.stride()), _native.strides4(v.stride()),
            dtype_code, 1 if causal else 0, float(scale), int(kv_begin), int(kv_end), int(n_split),
            status.data_ptr(), stream,
        )
        if rc != _native.TA_OK:
            _raise_for(lib, rc)
        if _sync_mode() in ("post", "strict"):
            check_device_status(q.device)
    return o_part, lse_part


def run_lse_combine(o_part, lse_part, *, out_dtype, head_dim: int | None = None,
                    return_lse: bool = False):
    """Merge split-KV partials (layout of run_sdpa_partial) on the GPU into o [B,H,S,D]
    of out_dtype (float16 / bfloat16 / float32) and, optionally, lse [B,H,S]."""
    torch_mod = _runtime.get_torch_module()
    lib = _runtime.get_native_library()
    n_split, batch, heads, seq_len, kdim = (int(x) for x in o_part.shape)
    o = torch_mod.empty((batch, heads, seq_len, kdim), dtype=out_dtype, device=o_part.device)
    lse = torch_mod.empty((batch, heads, seq_len), dtype=torch_mod.float32, device=o_part.device)
    code = _native.TA_DTYPE_F32 if out_dtype == torch_mod.float32 else _dtype_code(torch_mod, out_dtype)
    if o.numel() > 0:
        o_part = o_part.contiguous()
        lse_part = lse_part.contiguous()
        with torch_mod.cuda.device(o_part.device):
            stream = torch_mod.cuda.current_stream(o_part.device).cuda_stream
            rc = lib.ta_lse_combine(o_part.data_ptr(), lse_part.data_ptr(), n_split, batch, heads,
                                    seq_len, kdim, o.data_ptr(), _native.strides4(o.stride()),
                                    code, lse.data_ptr() if return_lse else None, stream)
            if rc != _native.TA_OK:
                _raise_for(lib, rc)
    if head_dim is not None and head_dim != kdim:
        o = o[..., :head_dim]
    return (o, lse) if return_lse else o
