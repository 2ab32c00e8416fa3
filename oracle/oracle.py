"""CPU oracle of the SDPA forward — TEST INFRASTRUCTURE ONLY.

Used by tests/ (parity checker), __graft_entry__.smoke() (checker) and bench.py
(timed CPU baseline / reference arm). The product package tiledattention_b200 never
imports this module.

Two independent restatements of the reference algorithm
(src/tiledattention/kernels/flash_fwd.py:400-444: scale, top-left causal + bounds
mask, softmax, normalise; same maths as the reference's math-path baselines
benchmark-gb10/run_study.py:249-271,304-335):
  * sdpa_numpy: numpy float64, blocked over query rows;
  * sdpa_c:     the C library oracle/_build/libsdpa_oracle.so (float64 for parity,
                float32 for the timed CPU baseline), multi-threaded.
Both take fp16/bf16 tensors or arrays, upcast them exactly and return float32.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libsdpa_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the C oracle with its Makefile (gcc, no GPU needed)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        lib = ctypes.CDLL(LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        lib.ta_oracle_sdpa_f64.argtypes = [fp, fp, fp, fp, fp] + [ctypes.c_int] * 4 + [
            ctypes.c_double, ctypes.c_int, ctypes.c_int]
        lib.ta_oracle_sdpa_f64.restype = None
        lib.ta_oracle_sdpa_f32.argtypes = [fp, fp, fp, fp, fp] + [ctypes.c_int] * 4 + [
            ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.ta_oracle_sdpa_f32.restype = None
        lib.ta_oracle_threads.restype = ctypes.c_int
        lib.ta_oracle_set_threads.argtypes = [ctypes.c_int]
        _lib = lib
    return _lib


def _to_f32(x) -> np.ndarray:
    """torch tensor (any float dtype, any device) or ndarray -> contiguous float32 ndarray."""
    if hasattr(x, "detach"):
        x = x.detach().float().cpu().contiguous().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def sdpa_numpy(q, k, v, *, causal: bool, scale: float, block: int = 256,
               return_lse: bool = False, kv_range: tuple[int, int] | None = None):
    """float64 restatement; q,k,v [B,H,S,D]. Returns float32 [B,H,S,D] (and lse [B,H,S]).
    kv_range=(lo, hi) restricts the keys to [lo, hi) (split-KV partial state); rows with no
    valid key then give o = 0 and lse = -inf."""
    q, k, v = (_to_f32(t).astype(np.float64) for t in (q, k, v))
    B, H, S, D = q.shape
    out = np.empty((B, H, S, D), dtype=np.float64)
    lse = np.empty((B, H, S), dtype=np.float64)
    cols = np.arange(S)
    for r0 in range(0, S, block):
        r1 = min(S, r0 + block)
        s = np.einsum("bhrd,bhcd->bhrc", q[:, :, r0:r1], k) * scale
        valid = np.ones((r1 - r0, S), dtype=bool)
        if causal:
            valid &= cols[None, :] <= np.arange(r0, r1)[:, None]
        if kv_range is not None:
            valid &= (cols[None, :] >= kv_range[0]) & (cols[None, :] < kv_range[1])
        s = np.where(valid, s, -np.inf)
        m = s.max(axis=-1, keepdims=True)
        m_safe = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(s - m_safe)
        l = p.sum(axis=-1, keepdims=True)
        with np.errstate(invalid="ignore", divide="ignore"):
            out[:, :, r0:r1] = np.where(l > 0, np.einsum("bhrc,bhcd->bhrd", p, v) / l, 0.0)
            lse[:, :, r0:r1] = np.where(l > 0, m_safe + np.log(l), -np.inf)[..., 0]
    if return_lse:
        return out.astype(np.float32), lse.astype(np.float32)
    return out.astype(np.float32)


def sdpa_c(q, k, v, *, causal: bool, scale: float, precision: str = "f64",
           rows: tuple[int, int] | None = None, return_lse: bool = False, threads: int = 0):
    """C oracle; q,k,v [B,H,S,D]. rows=(r0,r1) restricts the computed query rows of
    every head (the rest of the output is NaN). precision 'f64' (parity) or 'f32'."""
    lib = load()
    q, k, v = (_to_f32(t) for t in (q, k, v))
    B, H, S, D = q.shape
    out = np.full((B, H, S, D), np.nan, dtype=np.float32)
    lse = np.full((B, H, S), np.nan, dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, S)
    fp = ctypes.POINTER(ctypes.c_float)
    args = [t.ctypes.data_as(fp) for t in (q, k, v, out, lse)]
    lib.ta_oracle_set_threads(int(threads))
    fn = lib.ta_oracle_sdpa_f64 if precision == "f64" else lib.ta_oracle_sdpa_f32
    fn(*args, B * H, S, D, 1 if causal else 0, float(scale), int(r0), int(r1))
    return (out, lse) if return_lse else out


def oracle_threads() -> int:
    return int(load().ta_oracle_threads())


def attention_forward_flops(B: int, H: int, S: int, D: int, causal: bool) -> float:
    """FLOP count of one forward, the reference's formula
    (benchmark-gb10/run_study.py:95-112): causal 2*B*H*S*(S+1)*D, else 4*B*H*S^2*D."""
    if causal:
        return 2.0 * B * H * S * (S + 1) * D
    return 4.0 * B * H * S * S * D


def approximate_bytes(B: int, H: int, S: int, D: int, elem_bytes: int) -> float:
    """Algorithmic HBM bytes (q, k, v read + o written), run_study.py:130-148."""
    return 4.0 * B * H * S * D * elem_bytes
