"""Pins the CPU oracle to the reference: every golden fixture's expected output was
produced by the reference's own standard_eager_attention (run_study.py:304-335) and
torch SDPA in float64 (tests/golden/make_golden.py). CPU only."""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def load_case(path):
    z = np.load(path)
    dt = torch.bfloat16 if str(z["dtype"]) == "bfloat16" else torch.float16
    q, k, v = (torch.from_numpy(z[n].copy()).view(dt) for n in ("q", "k", "v"))
    return q, k, v, bool(z["causal"]), float(z["scale"]), z["expected"], z["expected_reference_eager"]


def test_fixtures_present():
    assert len(GOLDEN) >= 5


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_golden(path):
    q, k, v, causal, scale, expected, eager = load_case(path)
    assert np.abs(expected - eager).max() < 1e-5  # reference math path vs torch SDPA
    o64 = oracle.sdpa_c(q, k, v, causal=causal, scale=scale, precision="f64")
    onp = oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale)
    o32 = oracle.sdpa_c(q, k, v, causal=causal, scale=scale, precision="f32")
    assert np.abs(o64 - expected).max() < 2e-6
    assert np.abs(onp - expected).max() < 2e-6
    assert np.abs(o32 - expected).max() < 5e-5


@pytest.mark.parametrize("path", GOLDEN[:2], ids=[os.path.basename(p) for p in GOLDEN[:2]])
def test_oracle_row_sampling_and_lse(path):
    q, k, v, causal, scale, expected, _ = load_case(path)
    S = q.shape[2]
    out, lse = oracle.sdpa_c(q, k, v, causal=causal, scale=scale, rows=(S // 2, S),
                             return_lse=True)
    assert np.isnan(out[:, :, : S // 2]).all()
    assert np.abs(out[:, :, S // 2:] - expected[:, :, S // 2:]).max() < 2e-6
    _, lse_np = oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale, return_lse=True)
    assert np.abs(lse[:, :, S // 2:] - lse_np[:, :, S // 2:]).max() < 1e-5


def test_flop_formula_matches_reference():
    # run_study.py:95-112
    assert oracle.attention_forward_flops(8, 32, 4096, 128, True) == 2 * 256 * 4096 * 4097 * 128
    assert oracle.attention_forward_flops(1, 8, 1024, 64, False) == 4 * 8 * 1024 * 1024 * 64
    assert oracle.approximate_bytes(1, 8, 1024, 64, 2) == 4 * 8 * 1024 * 64 * 2
