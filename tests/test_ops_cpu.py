"""The torch operator registration (tiledattention_b200.ops) without a GPU: the ops exist
under torch.ops.tiledattention_b200 with the documented schema, and their fake (meta)
implementations give the output shapes and dtypes."""

import os

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


def test_native_ops_are_the_cpp_registration():
    # with the native launcher built (in-tree), the operators are the C++ ones
    from tiledattention_b200 import ops

    assert ops.NATIVE_OPS
    q = torch.empty(1, 2, 10, 100, dtype=torch.float16, device="meta")
    o_p, lse = torch.ops.tiledattention_b200.sdpa_fwd_partial(q, q, q, True, 0.1, 0, 10, 2)
    assert o_p.shape == (2, 1, 2, 10, 100) and lse.shape == (2, 1, 2, 10)


def test_python_registration_when_launcher_disabled():
    import subprocess
    import sys

    code = (
        "import torch, tiledattention_b200.ops as ops\n"
        "assert not ops.NATIVE_OPS\n"
        "q = torch.empty(2, 3, 100, 96, dtype=torch.bfloat16, device='meta')\n"
        "o = torch.ops.tiledattention_b200.sdpa_fwd(q, q, q, True, 0.1)\n"
        "assert o.shape == q.shape\n"
        "s = str(torch.ops.tiledattention_b200.sdpa_fwd.default._schema)\n"
        "assert 'sdpa_fwd(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> Tensor' in s\n"
    )
    env = dict(os.environ, TILEDATTN_FAST_LAUNCH="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr
