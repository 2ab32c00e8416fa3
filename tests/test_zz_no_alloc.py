"""The allocation-free split-KV entry point, ta_sdpa_fwd_split_noalloc, called through the
C ABI. It exists for callers that cannot allocate device memory around the attention call
(a plugin given only its inputs and outputs by a host that owns the GPU memory, or a
latency-critical loop where cudaMalloc could synchronise or fail); its slice partials live
in a fixed array inside the library instead of a per-call buffer.

The tests compare it, on two calls in a row (the second reuses the scratch array the first
one filled), with the regular entry point ta_sdpa_fwd on the same inputs and with the
float64 CPU oracle, within the tolerance of the parity tests; one case fills the array to
within 2 KB of its 64 MiB limit and the next row count is rejected. They live in their own
file named to be collected last."""

import math

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
RTOL = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -8}


def _strides(t):
    from tiledattention_b200 import _native

    return _native.strides4(t.stride())


def test_noalloc_split_matches_regular_entry_point_twice():
    from tiledattention_b200 import _native

    lib = _native.load_library()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    cases = [
        (torch.bfloat16, 1, 4, 3001, 128, True, 4),   # ragged S, causal
        (torch.float16, 2, 2, 1000, 64, False, 3),     # non-causal, head dim 64
        (torch.bfloat16, 1, 2, 700, 256, True, 2),     # head dim 256 (shared-K/V kernel)
        (torch.float16, 1, 3, 500, 96, False, 2),      # head dim 96, no padded copies
    ]
    for call in range(2):
        for dtype, B, H, S, D, causal, n_split in cases:
            g = torch.Generator().manual_seed(100 * call + S)
            q, k, v = (torch.randn(B, H, S, D, generator=g).to(dtype).to(dev) for _ in range(3))
            code = _native.TA_DTYPE_BF16 if dtype == torch.bfloat16 else _native.TA_DTYPE_F16
            scale = 1.0 / math.sqrt(D)
            o_ref = torch.empty_like(q)
            o_new = torch.full_like(q, float("nan"))
            rc = lib.ta_sdpa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_ref.data_ptr(), None,
                                 B, H, S, D, _strides(q), _strides(k), _strides(v), _strides(o_ref),
                                 code, int(causal), scale, None, stream)
            assert rc == 0, _native.last_error(lib)
            rc = lib.ta_sdpa_fwd_split_noalloc(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), o_new.data_ptr(), None,
                B, H, S, D, _strides(q), _strides(k), _strides(v), _strides(o_new),
                code, int(causal), scale, n_split, None, stream)
            assert rc == 0, _native.last_error(lib)
            torch.cuda.synchronize(dev)
            ref, got = o_ref.float(), o_new.float()
            assert torch.isfinite(got).all()
            bound = TOL[dtype] + RTOL[dtype] * ref.abs()
            assert float(((got - ref).abs() - bound).max()) <= 0, float((got - ref).abs().max())
            exact = torch.from_numpy(oracle.sdpa_c(q, k, v, causal=causal, scale=scale))
            got = got.cpu()
            bound = TOL[dtype] + RTOL[dtype] * exact.abs()
            assert float(((got - exact).abs() - bound).max()) <= 0, float((got - exact).abs().max())


def test_noalloc_split_rejects_oversized_problem():
    from tiledattention_b200 import _native

    lib = _native.load_library()
    st = _native.strides4([16 * 65536 * 128, 65536 * 128, 128, 1])
    # 8 slices x 16 heads x 65536 rows x 129 floats is far beyond the 64 MiB array
    rc = lib.ta_sdpa_fwd_split_noalloc(16, 16, 16, 16, None, 1, 16, 65536, 128, st, st, st, st,
                                       _native.TA_DTYPE_BF16, 1, 0.1, 8, None, None)
    assert rc == _native.TA_ERR_INVALID_ARGUMENT
    assert "64 MiB" in _native.last_error(lib)


def test_noalloc_split_at_the_size_limit():
    """n_split*B*H*S*(D+1)*4 bytes just below 64 MiB (2 slices x 2 heads x 32513 rows x 129
    floats = 67106832 bytes): the lse region after the partial outputs ends 2032 bytes
    before the end of the array. The result must match ta_sdpa_fwd and, on sampled rows,
    the oracle; one more row (67108896 bytes) is rejected."""
    from tiledattention_b200 import _native

    lib = _native.load_library()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    B, H, D, n_split, S = 1, 2, 128, 2, 32513
    assert n_split * B * H * S * (D + 1) * 4 <= 64 << 20 < n_split * B * H * (S + 1) * (D + 1) * 4
    g = torch.Generator().manual_seed(4242)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    scale = 1.0 / math.sqrt(D)
    code = _native.TA_DTYPE_BF16
    o_ref = torch.empty_like(qd)
    rc = lib.ta_sdpa_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o_ref.data_ptr(), None,
                         B, H, S, D, _strides(qd), _strides(kd), _strides(vd), _strides(o_ref),
                         code, 1, scale, None, stream)
    assert rc == 0, _native.last_error(lib)
    lse = torch.full((B * H * S,), float("nan"), dtype=torch.float32, device=dev)
    for _ in range(2):
        o_new = torch.full_like(qd, float("nan"))
        rc = lib.ta_sdpa_fwd_split_noalloc(
            qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o_new.data_ptr(), lse.data_ptr(),
            B, H, S, D, _strides(qd), _strides(kd), _strides(vd), _strides(o_new),
            code, 1, scale, n_split, None, stream)
        assert rc == 0, _native.last_error(lib)
        torch.cuda.synchronize(dev)
        ref, got = o_ref.float(), o_new.float()
        assert torch.isfinite(got).all() and torch.isfinite(lse).all()
        bound = TOL[torch.bfloat16] + RTOL[torch.bfloat16] * ref.abs()
        assert float(((got - ref).abs() - bound).max()) <= 0
    rows = (S - 64, S)
    exact, exact_lse = oracle.sdpa_c(q, k, v, causal=True, scale=scale, rows=rows, return_lse=True)
    exact = torch.from_numpy(exact)[:, :, rows[0]:rows[1]]
    got = o_new.float().cpu()[:, :, rows[0]:rows[1]]
    bound = TOL[torch.bfloat16] + RTOL[torch.bfloat16] * exact.abs()
    assert float(((got - exact).abs() - bound).max()) <= 0
    got_lse = lse.cpu().view(B, H, S)[:, :, rows[0]:rows[1]]
    exact_lse = torch.from_numpy(exact_lse).view(B, H, S)[:, :, rows[0]:rows[1]]
    assert float((got_lse - exact_lse).abs().max()) < 1e-3
    rc = lib.ta_sdpa_fwd_split_noalloc(
        qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o_new.data_ptr(), None,
        B, H, S + 1, D, _strides(qd), _strides(kd), _strides(vd), _strides(o_new),
        code, 1, scale, n_split, None, stream)
    assert rc == _native.TA_ERR_INVALID_ARGUMENT
    assert "64 MiB" in _native.last_error(lib)
