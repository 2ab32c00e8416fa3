"""Output canaries: the kernels write exactly their output and nothing around it.

The output of ta_sdpa_fwd is placed as a window inside a larger buffer filled with a
sentinel (rows before and after each (b,h) block, columns after the head dim, whole heads
between), passed through the C ABI with the buffer's strides. After the call the window must
equal the output of a plain contiguous call and every other element must still hold the
sentinel: ragged S (rows >= S clipped by the TMA store), head dims that run on a wider
kernel tile (96 on the 128 kernel, 200 on the 256 kernel: columns past D never written), the
shared-K/V kernel, the fp32 partials of ta_sdpa_fwd_partial and the lse array."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SENTINEL = 1234.5


def _inputs(B, H, S, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, H, S, D, generator=g).to(dtype).to(DEV) for _ in range(3))


@pytest.mark.parametrize("B,H,S,D,causal", [
    (2, 3, 1000, 128, True),    # persistent kernel, ragged S (TMA store clips rows)
    (1, 2, 300, 96, False),     # persistent kernel on the 128 tile, columns 96-127 not written
    (1, 2, 257, 64, True),
    (1, 2, 300, 200, True),     # shared-K/V kernel on the 256 tile
    (1, 16, 32768, 128, False), # shared-K/V kernel at D=128 (B*H*S^2 = 2^34)
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_output_window_only(B, H, S, D, causal, dtype):
    from tiledattention_b200 import _native
    from tiledattention_b200.launch import _status_word

    lib = _native.load_library()
    q, k, v = _inputs(B, H, S, D, dtype, S + D)
    code = _native.TA_DTYPE_BF16 if dtype == torch.bfloat16 else _native.TA_DTYPE_F16
    stream = torch.cuda.current_stream().cuda_stream
    status = _status_word(torch, DEV)
    scale = 1.0 / math.sqrt(D)

    def call(o, lse):
        st = _native.strides16(q.stride(), k.stride(), v.stride(), o.stride())
        rc = lib.ta_sdpa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr() if lse is not None else None, B, H, S, D,
                             st[0], st[1], st[2], st[3], code, int(causal), scale,
                             status.data_ptr(), stream)
        assert rc == 0, _native.last_error(lib)

    ref = torch.empty(B, H, S, D, dtype=dtype, device=DEV)
    ref_lse = torch.empty(B, H, S, device=DEV)
    call(ref, ref_lse)
    # window: 3 rows before / 5 after each (b,h) block, 24 spare columns, one spare head
    big = torch.full((B, H + 1, S + 8, D + 24), SENTINEL, dtype=dtype, device=DEV)
    o = big[:, 1:, 3:3 + S, :D]
    lse_big = torch.full((B * H * S + 64,), SENTINEL, device=DEV)
    lse = lse_big[32:32 + B * H * S].view(B, H, S)
    call(o, lse)
    torch.cuda.synchronize()
    from tiledattention_b200 import check_device_status

    check_device_status(DEV)
    assert torch.equal(o, ref)
    assert torch.equal(lse, ref_lse)
    mask = torch.ones_like(big, dtype=torch.bool)
    mask[:, 1:, 3:3 + S, :D] = False
    assert bool((big[mask] == SENTINEL).all()), "kernel wrote outside its output window"
    assert bool((lse_big[:32] == SENTINEL).all()) and bool((lse_big[32 + B * H * S:] ==
                                                              SENTINEL).all())


@pytest.mark.parametrize("D", [128, 96])
def test_partial_state_stays_in_its_arrays(D):
    from tiledattention_b200 import _native
    from tiledattention_b200.launch import _status_word

    lib = _native.load_library()
    B, H, S, n = 1, 2, 700, 3
    q, k, v = _inputs(B, H, S, D, torch.bfloat16, D)
    stream = torch.cuda.current_stream().cuda_stream
    status = _status_word(torch, DEV)
    o_elems, l_elems = n * B * H * S * D, n * B * H * S
    o_big = torch.full((o_elems + 64,), SENTINEL, device=DEV)
    l_big = torch.full((l_elems + 64,), SENTINEL, device=DEV)
    o_part, lse_part = o_big[:o_elems], l_big[:l_elems]
    rc = lib.ta_sdpa_fwd_partial(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_part.data_ptr(),
                                 lse_part.data_ptr(), B, H, S, D, _native.strides4(q.stride()),
                                 _native.strides4(k.stride()), _native.strides4(v.stride()),
                                 _native.TA_DTYPE_BF16, 1, D ** -0.5, 0, S, n,
                                 status.data_ptr(), stream)
    assert rc == 0, _native.last_error(lib)
    torch.cuda.synchronize()
    assert bool((o_big[o_elems:] == SENTINEL).all()) and bool((l_big[l_elems:] == SENTINEL).all())
    assert not bool((o_part == SENTINEL).any()) and not bool((lse_part == SENTINEL).any())
