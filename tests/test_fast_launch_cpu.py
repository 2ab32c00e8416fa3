"""The one-call host launcher (csrc/fast_launch.cpp) builds, loads and binds to the native
library without a GPU, and declines every input it cannot take (returning None, having
launched nothing), so the Python path raises the reference's errors for them."""

import os

import pytest
import torch

from tiledattention_b200 import _native, build


@pytest.fixture(scope="module")
def fast():
    build.build_fast_launch()
    lib = _native.load_library()
    mod = _native.load_fast_launch(lib)
    if mod is None:
        pytest.fail("fast launcher did not load: " + build.fast_launch_path())
    return mod


def test_built_in_tree(fast):
    assert os.path.exists(build.fast_launch_path())
    assert os.path.dirname(build.fast_launch_path()) == os.path.dirname(_native.LIB_PATH)


def test_declines_host_tensors(fast):
    q = torch.randn(1, 2, 64, 64, dtype=torch.float16)
    before = fast.launches()
    assert fast.launch(q, q, q, True, -1.0, False) is None
    assert fast.launch(q, q, q, False, 0.125, True) is None
    assert fast.launches() == before


@pytest.mark.parametrize("args", [
    ("x", "y", "z", True, 1.0, False),       # not tensors
    (None, None, None, 1, 1.0, False),       # non-bool causal
    (None, None, None, True, 1, False),      # non-float scale
    (None, None, None, True, -2.0, False),   # non-positive scale other than the default code
    (None, None, None, True, float("nan"), False),
])
def test_declines_bad_arguments(fast, args):
    q = torch.randn(1, 1, 8, 64, dtype=torch.float16)
    args = tuple(q if a is None else a for a in args)
    assert fast.launch(*args) is None
    assert fast.launch(q, q, q) is None  # wrong arity


def test_api_guards_before_the_launcher(monkeypatch):
    # -1.0 is the launcher's code for the default scale: a caller passing it (or any
    # non-positive or non-float scale) must not reach the launcher and gets the reference's
    # InvalidShapeError (sdpa.py:37-40).
    from tiledattention_b200 import InvalidShapeError, _runtime, sdpa

    calls = []

    class Stub:
        @staticmethod
        def launch(*a):
            calls.append(a)
            return None

    monkeypatch.setattr(_native, "_fast", Stub)
    monkeypatch.setattr(_runtime, "_runtime_ready", True)
    q = torch.randn(1, 1, 8, 64, dtype=torch.float16)
    for bad in (-1.0, 0.0, -3.0, float("nan")):
        with pytest.raises(InvalidShapeError):
            sdpa(q, q, q, scale=bad)
    assert calls == []
    monkeypatch.setenv("TILEDATTN_SYNC_MODE", "strict")
    with pytest.raises(Exception):
        sdpa(q, q, q)
    assert calls == []
    monkeypatch.delenv("TILEDATTN_SYNC_MODE")
    with pytest.raises(Exception):
        sdpa(q, q, q, causal=True, scale=0.5)
    assert len(calls) == 1 and calls[0][3:] == (True, 0.5, False)
