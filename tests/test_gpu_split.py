"""Split-KV path on the GPU: per-slice partial states (ta_sdpa_fwd_partial) against the
float64 oracle restricted to the same key range, the on-GPU log-sum-exp merge
(ta_lse_combine) through sdpa_split_kv against full attention, and the lse output.
Tolerances: partial states are fp32 (atol 2e-3 on o for 16-bit inputs, 1e-3 on lse);
merged outputs use the bound of test_gpu_parity (atol + rtol*|ref|)."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
RTOL = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -8}
# lse = m + log(l) with l summed from the 16-bit weights the P.V MMA uses: relative error
# of l up to about one 16-bit ulp, i.e. 2^-8 (bf16) / 2^-10 (fp16) in log space.
LSE_TOL = {torch.float16: 1e-3, torch.bfloat16: 4e-3}


def _inputs(B, H, S, D, dtype, seed, sigma=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, S, D, generator=g) * sigma).to(dtype)
    k = (torch.randn(B, H, S, D, generator=g) * sigma).to(dtype)
    v = torch.randn(B, H, S, D, generator=g).to(dtype)
    return q, k, v


def _bound_ok(got, ref, dtype):
    diff = (got - ref).abs()
    return float((diff - (TOL[dtype] + RTOL[dtype] * ref.abs())).max()) <= 0, float(diff.max())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S,n_split", [(1000, 3), (2048, 8), (300, 1), (129, 4)])
def test_split_kv_matches_full(S, n_split, causal, D, dtype):
    import tiledattention_b200 as ta

    q, k, v = _inputs(1, 3, S, D, dtype, S + n_split)
    dev = torch.device("cuda:0")
    o, lse = ta.sdpa_split_kv(q.to(dev), k.to(dev), v.to(dev), causal=causal, n_split=n_split,
                              return_lse=True)
    ta.check_device_status(dev)
    ref, ref_lse = oracle.sdpa_numpy(q, k, v, causal=causal, scale=D ** -0.5, return_lse=True)
    ok, err = _bound_ok(o.float().cpu(), torch.from_numpy(ref), dtype)
    assert ok, err
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_TOL[dtype]


@pytest.mark.parametrize("D", [40, 96, 100, 200])
@pytest.mark.parametrize("causal", [False, True])
def test_split_kv_other_head_dims(D, causal):
    """Head dims that are not 64/128/256: multiples of 8 keep their own head dim in the
    split-KV state (no padded copies, merged by the run-time-D merge kernel); others are
    padded to the next native size and sliced."""
    import tiledattention_b200 as ta

    dtype = torch.float16
    q, k, v = _inputs(1, 3, 700, D, dtype, D)
    dev = torch.device("cuda:0")
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    o, lse = ta.sdpa_split_kv(qd, kd, vd, causal=causal, n_split=3, return_lse=True)
    o_p, l_p = ta.sdpa_partial(qd, kd, vd, causal=causal, n_split=3)
    ta.check_device_status(dev)
    assert o.shape == q.shape and o_p.shape[-1] == D
    ref, ref_lse = oracle.sdpa_numpy(q, k, v, causal=causal, scale=D ** -0.5, return_lse=True)
    ok, err = _bound_ok(o.float().cpu(), torch.from_numpy(ref), dtype)
    assert ok, err
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_TOL[dtype]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("kv", [(0, 128), (128, 700), (256, 257), (640, 1000)])
def test_partial_state_matches_oracle(kv, causal):
    import tiledattention_b200 as ta

    S, D, dtype = 1000, 128, torch.bfloat16
    q, k, v = _inputs(2, 2, S, D, dtype, 5)
    dev = torch.device("cuda:0")
    o_p, l_p = ta.sdpa_partial(q.to(dev), k.to(dev), v.to(dev), causal=causal,
                               kv_begin=kv[0], kv_end=kv[1])
    ta.check_device_status(dev)
    ref, ref_lse = oracle.sdpa_numpy(q, k, v, causal=causal, scale=D ** -0.5, return_lse=True,
                                     kv_range=kv)
    got_l = l_p[0].cpu().numpy()
    assert np.array_equal(np.isinf(got_l), np.isinf(ref_lse))  # empty rows agree
    fin = np.isfinite(ref_lse)
    assert np.abs(got_l[fin] - ref_lse[fin]).max() < LSE_TOL[dtype]
    assert np.abs(o_p[0].cpu().numpy() - ref).max() < 1.5e-2  # P rounded to bf16 in the MMA


def test_lse_output_of_sdpa_with_lse():
    import tiledattention_b200 as ta

    q, k, v = _inputs(1, 4, 777, 64, torch.float16, 9, sigma=4.0)
    dev = torch.device("cuda:0")
    o, lse = ta.sdpa_with_lse(q.to(dev), k.to(dev), v.to(dev), causal=True)
    ta.check_device_status(dev)
    _, ref_lse = oracle.sdpa_numpy(q, k, v, causal=True, scale=1 / 8, return_lse=True)
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_TOL[torch.float16]


def test_split_kv_long_context_sampled_rows():
    """Config-5 shape family at reduced heads: S=65536, D=128, bf16, causal; rows sampled."""
    import tiledattention_b200 as ta

    S, D = 65536, 128
    q, k, v = _inputs(1, 1, S, D, torch.bfloat16, 65)
    dev = torch.device("cuda:0")
    o = ta.sdpa_split_kv(q.to(dev), k.to(dev), v.to(dev), causal=True, n_split=8)
    o_full = ta.sdpa(q.to(dev), k.to(dev), v.to(dev), causal=True)
    ta.check_device_status(dev)
    rows = (S - 64, S)
    ref = torch.from_numpy(oracle.sdpa_c(q, k, v, causal=True, scale=D ** -0.5, rows=rows))
    for out in (o, o_full):
        ok, err = _bound_ok(out.float().cpu()[:, :, rows[0]:rows[1]], ref[:, :, rows[0]:rows[1]],
                            torch.bfloat16)
        assert ok, err
