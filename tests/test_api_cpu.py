"""Host-side behaviour of the drop-in API, CPU only (fake torch, as the reference's
own tests do: tests/test_errors.py, tests/test_sdpa_shapes.py, tests/test_imports.py,
tests/test_tiledattention.py of thisistaimur/TiledAttention)."""

from __future__ import annotations

from dataclasses import dataclass
from types import ModuleType

import pytest

import tiledattention_b200._runtime as runtime
import importlib

sdpa_mod = importlib.import_module("tiledattention_b200.sdpa")
from tiledattention_b200 import (
    DependencyError,
    DTypeNotSupportedError,
    InvalidShapeError,
    TiledAttentionError,
    UnsupportedPlatformError,
)
from tiledattention_b200._runtime import _reset_runtime_cache_for_tests, require_supported_runtime
from tiledattention_b200.sdpa import sdpa


@dataclass
class FakeTensor:
    shape: tuple
    dtype: object
    device: str
    is_cuda: bool

    @property
    def ndim(self) -> int:
        return len(self.shape)


def _fake_torch(*, cuda_available=True, capability=(10, 0)):
    torch_mod = ModuleType("torch")
    torch_mod.Tensor = FakeTensor
    torch_mod.float16 = object()
    torch_mod.bfloat16 = object()

    class FakeCuda:
        @staticmethod
        def is_available():
            return cuda_available

        @staticmethod
        def current_device():
            return 0

        @staticmethod
        def get_device_capability(_i):
            return capability

    torch_mod.cuda = FakeCuda()
    return torch_mod


@pytest.fixture
def fake_runtime(monkeypatch):
    def install(**kw):
        tm = _fake_torch(**kw)
        monkeypatch.setattr(runtime, "_get_torch_module", lambda: tm)
        monkeypatch.setattr(runtime, "_get_native_library", lambda: object())
        _reset_runtime_cache_for_tests()
        return tm

    yield install
    _reset_runtime_cache_for_tests()


def _t(tm, shape=(1, 2, 64, 64), dtype=None, device="cuda:0", is_cuda=True):
    return FakeTensor(shape=shape, dtype=dtype if dtype is not None else tm.float16,
                      device=device, is_cuda=is_cuda)


def test_import_and_version():
    import tiledattention
    import tiledattention_b200

    assert isinstance(tiledattention_b200.__version__, str) and tiledattention_b200.__version__
    assert tiledattention.__version__ == tiledattention_b200.__version__


def test_sdpa_stays_callable_after_submodule_import():
    # the reference's lazy import turns tiledattention.sdpa into a module after one call
    import tiledattention
    from tiledattention.sdpa import sdpa as f  # noqa: F401

    import tiledattention_b200.sdpa  # noqa: F401

    assert callable(tiledattention.sdpa)
    import tiledattention_b200

    assert callable(tiledattention_b200.sdpa)


def test_error_hierarchy():
    for cls in (UnsupportedPlatformError, InvalidShapeError, DTypeNotSupportedError, DependencyError):
        assert issubclass(cls, TiledAttentionError)


def test_runtime_no_cuda(fake_runtime):
    fake_runtime(cuda_available=False)
    with pytest.raises(UnsupportedPlatformError, match=r"requires CUDA \+ Blackwell GPU"):
        require_supported_runtime()


@pytest.mark.parametrize("cc", [(9, 0), (12, 0), (10, 3)])
def test_runtime_wrong_capability(fake_runtime, cc):
    fake_runtime(capability=cc)
    with pytest.raises(UnsupportedPlatformError, match=f"compute capability {cc[0]}.{cc[1]}"):
        require_supported_runtime()


def test_runtime_missing_native_library(monkeypatch):
    tm = _fake_torch()
    monkeypatch.setattr(runtime, "_get_torch_module", lambda: tm)
    from tiledattention_b200 import _native

    monkeypatch.setattr(_native, "LIB_PATH", "/nonexistent/libtiledattention_b200.so")
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.delenv("TILEDATTN_NATIVE_LIB", raising=False)
    _reset_runtime_cache_for_tests()
    with pytest.raises(DependencyError, match="native library"):
        require_supported_runtime()
    _reset_runtime_cache_for_tests()


def test_scalar_checks_come_first(fake_runtime):
    fake_runtime(cuda_available=False)
    with pytest.raises(InvalidShapeError, match="causal must be a bool"):
        sdpa(None, None, None, causal=1)
    for bad in (0, -1.0, "x", float("nan")):
        with pytest.raises(InvalidShapeError, match="scale must be a positive"):
            sdpa(None, None, None, scale=bad)
    with pytest.raises(UnsupportedPlatformError):
        sdpa(None, None, None)


def test_validates_rank(fake_runtime):
    tm = fake_runtime()
    q = _t(tm, shape=(1, 2, 64))
    with pytest.raises(InvalidShapeError, match=r"\[B, H, S, D\]"):
        sdpa(q, q, q)


def test_validates_not_tensor(fake_runtime):
    tm = fake_runtime()
    with pytest.raises(InvalidShapeError, match="q must be a torch.Tensor"):
        sdpa(object(), _t(tm), _t(tm))


def test_validates_cuda(fake_runtime):
    tm = fake_runtime()
    q = _t(tm, device="cpu", is_cuda=False)
    with pytest.raises(InvalidShapeError, match="CUDA tensor"):
        sdpa(q, q, q)


def test_validates_shape_match(fake_runtime):
    tm = fake_runtime()
    with pytest.raises(InvalidShapeError, match="matching shape"):
        sdpa(_t(tm), _t(tm, shape=(1, 2, 32, 64)), _t(tm))


def test_validates_same_device(fake_runtime):
    tm = fake_runtime()
    with pytest.raises(InvalidShapeError, match="same CUDA device"):
        sdpa(_t(tm), _t(tm, device="cuda:1"), _t(tm))


def test_validates_dtype(fake_runtime):
    tm = fake_runtime()
    q = _t(tm, dtype=object())
    with pytest.raises(DTypeNotSupportedError, match="float16"):
        sdpa(q, q, q)
    with pytest.raises(DTypeNotSupportedError, match="identical dtype"):
        sdpa(_t(tm), _t(tm, dtype=tm.bfloat16), _t(tm))


def test_valid_input_reaches_launcher(fake_runtime, monkeypatch):
    tm = fake_runtime()
    seen = {}

    def fake_launch(q, k, v, *, causal, scale, return_lse=False):
        seen.update(causal=causal, scale=scale, lse=return_lse)
        return "ok"

    monkeypatch.setattr(sdpa_mod, "run_sdpa_fwd", fake_launch)
    q = _t(tm)
    assert sdpa(q, q, q) == "ok"
    assert seen == {"causal": False, "scale": 0.125, "lse": False}
    assert sdpa(q, q, q, causal=True, scale=0.5) == "ok"
    assert seen["scale"] == 0.5 and seen["causal"] is True
    assert sdpa_mod.sdpa_with_lse(q, q, q) == "ok" and seen["lse"] is True


def test_padded_head_dim_policy():
    from tiledattention_b200.launch import padded_head_dim

    assert [padded_head_dim(d) for d in (1, 32, 64, 65, 96, 128, 129, 160, 256)] == [
        64, 64, 64, 128, 128, 128, 256, 256, 256]
    with pytest.raises(InvalidShapeError):
        padded_head_dim(257)


def test_state_head_dim_policy():
    from tiledattention_b200.launch import state_head_dim

    # split-KV state keeps multiples of 8 unpadded; other head dims take the padded size
    assert [state_head_dim(d) for d in (8, 64, 96, 100, 128, 160, 200, 248, 256, 1)] == [
        8, 64, 96, 128, 128, 160, 200, 248, 256, 64]
    with pytest.raises(InvalidShapeError):
        state_head_dim(257)


@pytest.mark.parametrize("bad", ["strcit", "sync", "POSTT"])
def test_unknown_sync_mode_raises(monkeypatch, bad):
    """An unknown TILEDATTN_SYNC_MODE raises the reference's ValueError
    (flash_fwd.py:814-818) instead of silently running asynchronously."""
    from tiledattention_b200 import launch

    monkeypatch.setenv("TILEDATTN_SYNC_MODE", bad)
    with pytest.raises(ValueError, match="Unsupported TILEDATTN_SYNC_MODE"):
        launch._sync_mode()
    for good in ("async", " Post ", "STRICT"):
        monkeypatch.setenv("TILEDATTN_SYNC_MODE", good)
        assert launch._sync_mode() == good.strip().lower()
