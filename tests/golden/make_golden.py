"""Generate the golden fixtures in tests/golden/ (run in a container that has the
reference checkout; the fixtures themselves are committed and need nothing else).

    python tests/golden/make_golden.py /path/to/TiledAttention

Expected outputs come from the reference's own math-path implementation,
standard_eager_attention (benchmark-gb10/run_study.py:304-335), extracted from the
reference source with ast and executed on CPU in float64 (run_study.py itself imports
matplotlib and the cuTile package, so it is not imported whole). They are
cross-checked against torch.nn.functional.scaled_dot_product_attention in float64,
the comparator of the reference's GPU test (tests/test_sdpa_correctness_small.py:37-39).
Inputs are drawn on the CPU from fixed seeds and stored as 16-bit bit patterns.
"""

from __future__ import annotations

import ast
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    # name, dtype, B, H, S, D, causal, seed, sigma_qk
    ("cfg1_fp16_causal", torch.float16, 1, 2, 64, 64, True, 0, 1.0),
    ("cfg1_fp16_noncausal", torch.float16, 1, 2, 64, 64, False, 0, 1.0),
    ("ragged_bf16_causal_sigma4", torch.bfloat16, 1, 2, 100, 128, True, 11, 4.0),
    ("ragged_fp16_noncausal", torch.float16, 2, 2, 33, 64, False, 12, 1.0),
    ("tile_edge_bf16_causal", torch.bfloat16, 1, 1, 257, 128, True, 13, 1.0),
]


def load_reference_eager(ref_root: str):
    path = os.path.join(ref_root, "benchmark-gb10", "run_study.py")
    tree = ast.parse(open(path).read(), filename=path)
    fn = next(n for n in tree.body
              if isinstance(n, ast.FunctionDef) and n.name == "standard_eager_attention")
    mod = ast.Module(body=[fn], type_ignores=[])
    ns = {"torch": torch, "math": math}
    exec(compile(mod, path, "exec"), ns)
    return ns["standard_eager_attention"]


def main(ref_root: str) -> None:
    eager = load_reference_eager(ref_root)
    for name, dtype, B, H, S, D, causal, seed, sigma in CASES:
        g = torch.Generator().manual_seed(seed)
        q = (torch.randn(B, H, S, D, generator=g) * sigma).to(dtype)
        k = (torch.randn(B, H, S, D, generator=g) * sigma).to(dtype)
        v = torch.randn(B, H, S, D, generator=g).to(dtype)
        q64, k64, v64 = (t.double() for t in (q, k, v))
        out_ref = eager(q64, k64, v64, causal=causal)
        out_sdpa = torch.nn.functional.scaled_dot_product_attention(
            q64, k64, v64, is_causal=causal)
        gap = float((out_ref - out_sdpa).abs().max())
        assert gap < 1e-5, (name, gap)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            q=q.view(torch.int16).numpy(), k=k.view(torch.int16).numpy(),
            v=v.view(torch.int16).numpy(),
            dtype=np.array("bfloat16" if dtype == torch.bfloat16 else "float16"),
            causal=np.array(causal), scale=np.array(1.0 / math.sqrt(D)),
            expected=out_sdpa.float().numpy(), expected_reference_eager=out_ref.float().numpy(),
        )
        print(f"{name}: eager-vs-sdpa gap {gap:.2e}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the TiledAttention checkout>")
    main(sys.argv[1])
