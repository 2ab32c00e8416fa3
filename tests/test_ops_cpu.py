"""The torch operator registration (tiledattention_b200.ops) without a GPU: the ops exist
under torch.ops.tiledattention_b200 with the documented schema, and their fake (meta)
implementations give the output shapes and dtypes."""

import torch

import tiledattention_b200.ops  # noqa: F401  (registers the ops)


def test_ops_registered_with_schema():
    op = torch.ops.tiledattention_b200.sdpa_fwd.default
    assert "sdpa_fwd(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> Tensor" in str(
        op._schema)
    part = torch.ops.tiledattention_b200.sdpa_fwd_partial.default
    assert "-> (Tensor, Tensor)" in str(part._schema)


def test_fake_shapes_on_meta_tensors():
    q = torch.empty(2, 3, 100, 96, dtype=torch.bfloat16, device="meta")
    o = torch.ops.tiledattention_b200.sdpa_fwd(q, q, q, True, 0.1)
    assert o.shape == q.shape and o.dtype == q.dtype and o.device.type == "meta"
    o_p, lse = torch.ops.tiledattention_b200.sdpa_fwd_partial(q, q, q, False, 0.1, 0, 100, 3)
    assert o_p.shape == (3, 2, 3, 100, 96) and o_p.dtype == torch.float32
    assert lse.shape == (3, 2, 3, 100) and lse.dtype == torch.float32
