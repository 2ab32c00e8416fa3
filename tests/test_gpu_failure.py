"""Failure detection without a GPU fault: a wait inside the kernel is made to run out (the
MMA warp waits on a barrier nothing arrives on, with a 2 ms limit). The kernel must record
the timeout in the device status word, stop every role, free its tensor memory and return;
the host must raise KernelError, and the next launch on the same context must succeed."""

import math

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


# D=64 runs the kernel build whose barrier waits carry a suspend-time hint (abort flag and
# clock checked every 4th try); D=128 the one without.
@pytest.mark.parametrize("d,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_bounded_wait_reports_and_context_survives(monkeypatch, d, dtype):
    import tiledattention_b200 as ta
    from tiledattention_b200 import _native

    monkeypatch.setenv("TILEDATTN_SYNC_MODE", "async")
    lib = _native.load_library()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 1000, d, generator=g).to(dtype) for _ in range(3))
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ta.check_device_status(dev)  # clean start
    lib.ta_debug_set_selftest(1, 2_000_000)
    try:
        ta.sdpa(qd, kd, vd, causal=True)
        # Every role's waits share the 2 ms limit, and the stalled MMA issuer starves the
        # others: whichever role's wait runs out first records the timeout (at D=128 the MMA
        # issuer, at D=64, whose waits check the clock only every few hints, often the
        # epilogue).
        with pytest.raises(ta.KernelError, match="wait timed out"):
            ta.check_device_status(dev)
    finally:
        lib.ta_debug_set_selftest(0, 0)
    ta.check_device_status(dev)  # the word was cleared by the raise above
    o = ta.sdpa(qd, kd, vd, causal=True)
    ta.check_device_status(dev)
    ref = oracle.sdpa_c(q, k, v, causal=True, scale=1 / math.sqrt(d))
    assert float((o.float().cpu() - torch.from_numpy(ref)).abs().max()) < 1e-2


def test_sync_mode_post_raises_on_timeout(monkeypatch):
    import tiledattention_b200 as ta
    from tiledattention_b200 import _native

    lib = _native.load_library()
    dev = torch.device("cuda:0")
    q = torch.randn(1, 1, 300, 64, device=dev, dtype=torch.float16)
    monkeypatch.setenv("TILEDATTN_SYNC_MODE", "post")
    lib.ta_debug_set_selftest(1, 2_000_000)
    try:
        with pytest.raises(ta.KernelError):
            ta.sdpa(q, q, q)
    finally:
        lib.ta_debug_set_selftest(0, 0)
    ta.sdpa(q, q, q)  # post mode: raises if anything is left over
