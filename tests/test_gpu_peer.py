"""The peer-exchange kernels on one GPU (ta_peer_barrier, ta_lse_merge_peers).

The merge only needs device addresses, so one GPU can stand in for a group: the "peers"'
states are separate local buffers. The merged rows must match the single-GPU combine
(ta_lse_combine) of the same states, land in every destination, honour row_base/out_rows,
and the barrier must (a) pass at once for a group of one and (b) give up after its time
limit when a peer never arrives (a flag that nothing sets), record TA_DEVSTAT_PEER_TIMEOUT,
make the merge after it write NaN, and leave the context usable."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _addr_array(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return arr, ctypes.addressof(arr)


def _states(S=1000, D=128, n=4, dtype=torch.bfloat16):
    from tiledattention_b200.sdpa import sdpa_partial

    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(2, 3, S, D, generator=g).to(dtype).to(dev) for _ in range(3))
    o_part, lse_part = sdpa_partial(q, k, v, causal=True, n_split=n)
    return q, o_part.contiguous(), lse_part.contiguous()


@pytest.mark.parametrize("D", [128, 96])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_merge_matches_combine_and_row_window(out_dtype, D):
    from tiledattention_b200 import _native
    from tiledattention_b200.launch import _status_word, run_lse_combine

    lib = _native.load_library()
    q, o_part, lse_part = _states(D=D)
    n, B, H, S, D_state = o_part.shape
    assert D_state == D  # multiples of 8 keep their own head dim in the state
    ref_o, ref_lse = run_lse_combine(o_part, lse_part, out_dtype=out_dtype, return_lse=True)
    o_srcs, o_a = _addr_array([o_part[i].data_ptr() for i in range(n)])
    l_srcs, l_a = _addr_array([lse_part[i].data_ptr() for i in range(n)])
    code = _native.TA_DTYPE_F32 if out_dtype == torch.float32 else _native.TA_DTYPE_BF16
    stream = torch.cuda.current_stream().cuda_stream
    status = _status_word(torch, q.device)
    # Two destinations, full rows.
    outs = [torch.full((B, H, S, D), 7.0, dtype=out_dtype, device=q.device) for _ in range(2)]
    lses = [torch.zeros(B, H, S, device=q.device) for _ in range(2)]
    d_keep, d_a = _addr_array([t.data_ptr() for t in outs])
    ld_keep, ld_a = _addr_array([t.data_ptr() for t in lses])
    rc = lib.ta_lse_merge_peers(o_a, l_a, n, B, H, S, D, 0, S, d_a, ld_a, 2,
                                _native.strides4(outs[0].stride()), S, 0, code,
                                status.data_ptr(), stream)
    assert rc == 0, lib.ta_last_error()
    torch.cuda.synchronize()
    for o, lse in zip(outs, lses):
        assert torch.equal(o, ref_o)
        assert torch.allclose(lse, ref_lse, atol=1e-5, rtol=0, equal_nan=True)
    # One destination holding only rows [300, 650), written at row 0.
    s0, s1 = 300, 650
    win = torch.zeros(B, H, s1 - s0, D, dtype=out_dtype, device=q.device)
    wl = torch.zeros(B, H, s1 - s0, device=q.device)
    w_keep, w_a = _addr_array([win.data_ptr()])
    wl_keep, wl_a = _addr_array([wl.data_ptr()])
    rc = lib.ta_lse_merge_peers(o_a, l_a, n, B, H, S, D, s0, s1, w_a, wl_a, 1,
                                _native.strides4(win.stride()), s1 - s0, s0, code,
                                status.data_ptr(), stream)
    assert rc == 0, lib.ta_last_error()
    torch.cuda.synchronize()
    assert torch.equal(win, ref_o[:, :, s0:s1])
    assert torch.allclose(wl, ref_lse[:, :, s0:s1], atol=1e-5, rtol=0)
    # Argument checks reject bad windows and too many sources.
    assert lib.ta_lse_merge_peers(o_a, l_a, n, B, H, S, D, s0, s1, w_a, wl_a, 1,
                                  _native.strides4(win.stride()), s1 - s0 - 1, s0, code,
                                  None, stream) == _native.TA_ERR_INVALID_ARGUMENT
    assert lib.ta_lse_merge_peers(o_a, l_a, 17, B, H, S, D, 0, S, d_a, None, 1,
                                  _native.strides4(outs[0].stride()), S, 0, code,
                                  None, stream) == _native.TA_ERR_INVALID_ARGUMENT


def test_barrier_group_of_one_passes():
    import tiledattention_b200 as ta
    from tiledattention_b200 import _native
    from tiledattention_b200.launch import _status_word

    lib = _native.load_library()
    dev = torch.device("cuda:0")
    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    keep, fa = _addr_array([flags.data_ptr()])
    status = _status_word(torch, dev)
    stream = torch.cuda.current_stream().cuda_stream
    for epoch in range(1, 4):
        assert lib.ta_peer_barrier(fa, 1, 0, epoch, 50_000_000, status.data_ptr(), stream) == 0
    ta.check_device_status(dev)
    assert int(flags[0].item()) == 3


def test_barrier_times_out_and_context_survives(monkeypatch):
    import tiledattention_b200 as ta
    from tiledattention_b200 import _native
    from tiledattention_b200.launch import _status_word

    monkeypatch.setenv("TILEDATTN_SYNC_MODE", "async")
    lib = _native.load_library()
    q, o_part, lse_part = _states(S=300, n=2)
    n, B, H, S, D = o_part.shape
    dev = q.device
    ta.check_device_status(dev)
    # Rank 0 of a group of two whose peer (a local buffer here) never arrives.
    flags = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(2)]
    keep, fa = _addr_array([f.data_ptr() for f in flags])
    status = _status_word(torch, dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.ta_peer_barrier(fa, 2, 0, 1, 20_000_000, status.data_ptr(), stream) == 0
    out = torch.zeros(B, H, S, D, dtype=torch.bfloat16, device=dev)
    o_keep, o_a = _addr_array([o_part[i].data_ptr() for i in range(n)])
    l_keep, l_a = _addr_array([lse_part[i].data_ptr() for i in range(n)])
    d_keep, d_a = _addr_array([out.data_ptr()])
    assert lib.ta_lse_merge_peers(o_a, l_a, n, B, H, S, D, 0, S, d_a, None, 1,
                                  _native.strides4(out.stride()), S, 0, _native.TA_DTYPE_BF16,
                                  status.data_ptr(), stream) == 0
    with pytest.raises(ta.KernelError, match="peer barrier timed out"):
        ta.check_device_status(dev)
    assert torch.isnan(out.float()).all()
    assert int(flags[1][0].item()) == 1  # our arrival was still published to the peer
    # The context is intact: a normal forward still runs and is finite.
    o = ta.sdpa(q, q, q, causal=True)
    ta.check_device_status(dev)
    assert math.isfinite(float(o.float().abs().max()))
