"""Host-side multi-rank logic on CPU: pair sharding, zig-zag key slices, the log-sum-exp
merge, and the merge across ranks over gloo (world size 2), checked against the float64
oracle; plus failure detection on gloo ranks (no GPU involved): a rank that never joins, a
rank that raises, a rank that arrives after the process-group timeout, and ranks whose
shards differ in size."""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from tiledattention_b200.distributed import (
    lse_merge,
    merge_across_ranks,
    shard_pairs,
    zigzag_key_ranges,
)


def test_shard_pairs_partition():
    for n, w in [(256, 1), (256, 8), (255, 8), (3, 8), (16, 3)]:
        seen = []
        for r in range(w):
            a, c = shard_pairs(n, w, r)
            seen += list(range(a, a + c))
        assert seen == list(range(n))


@pytest.mark.parametrize("S,world", [(65536, 8), (4096, 2), (1000, 4), (129, 2), (64, 8)])
def test_zigzag_ranges_partition_and_balance(S, world):
    cover = []
    work = []
    for r in range(world):
        rr = zigzag_key_ranges(S, world, r)
        assert all(lo % 128 == 0 and lo < hi for lo, hi in rr)
        cover += [x for lo, hi in rr for x in range(lo, hi)]
        # causal work of a key range: number of (row, key) pairs with key <= row
        work.append(sum(sum(S - key for key in range(lo, hi)) for lo, hi in rr))
    assert sorted(cover) == list(range(S))
    if S >= 128 * 2 * world:
        assert max(work) / min(work) < 1.1


def _inputs(B, H, S, D, seed):
    g = np.random.default_rng(seed)
    return [g.standard_normal((B, H, S, D)).astype(np.float32) for _ in range(3)]


@pytest.mark.parametrize("causal", [False, True])
def test_lse_merge_equals_full_attention(causal):
    q, k, v = _inputs(1, 2, 300, 64, 0)
    scale = 0.125
    full, full_lse = oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale, return_lse=True)
    cuts = [0, 37, 128, 129, 300]
    parts = [oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale, return_lse=True,
                               kv_range=(a, b)) for a, b in zip(cuts[:-1], cuts[1:])]
    o, lse = lse_merge(torch.tensor(np.stack([p[0] for p in parts])),
                       torch.tensor(np.stack([p[1] for p in parts])))
    assert np.abs(o.numpy() - full).max() < 1e-5
    assert np.abs(lse.numpy() - full_lse).max() < 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _merge_worker(rank, world, port, causal, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _inputs(1, 2, 700, 64, 1)
        scale = 1 / 8
        os_, ls = [], []
        for lo, hi in zigzag_key_ranges(700, world, rank):
            o, l = oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale, return_lse=True,
                                     kv_range=(lo, hi))
            os_.append(o)
            ls.append(l)
        o_loc, l_loc = lse_merge(torch.tensor(np.stack(os_)), torch.tensor(np.stack(ls)))
        o, lse = merge_across_ranks(o_loc, l_loc)
        full, full_lse = oracle.sdpa_numpy(q, k, v, causal=causal, scale=scale, return_lse=True)
        out_q.put((rank, float(np.abs(o.numpy() - full).max()),
                   float(np.abs(lse.numpy() - full_lse).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_merge_across_two_gloo_ranks(causal):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_merge_worker, args=(r, world, PORTS[causal], causal, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(out_q.get(timeout=10) for _ in range(world))
    for _, err_o, err_l in res:
        assert err_o < 1e-5 and err_l < 1e-4


PORTS = {False: _free_port(), True: _free_port()}


def _late_worker(rank, world, port, out_q):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # this rank fails between steps: it leaves without joining the merge
        dist.destroy_process_group()
        out_q.put((rank, "left"))
        return
    try:
        merge_across_ranks(torch.zeros(2, 4, 8), torch.zeros(2, 4))
        out_q.put((rank, "no error"))
    except Exception as exc:  # the collective must fail, not hang
        out_q.put((rank, f"error: {type(exc).__name__}"))


def test_rank_that_never_joins_is_detected():
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_late_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = dict(out_q.get(timeout=10) for _ in range(2))
    assert res[1] == "left"
    assert res[0].startswith("error")


def test_row_share_partitions_rows():
    """The peer-memory merge's per-rank query-row shares tile [0, S) exactly, in rank order,
    with sizes differing by at most one."""
    from tiledattention_b200.distributed import row_share

    for seq_len in (1, 7, 128, 1000, 65536):
        for world in (1, 2, 3, 4, 8):
            shares = [row_share(seq_len, world, r) for r in range(world)]
            assert shares[0][0] == 0 and shares[-1][1] == seq_len
            for (a0, a1), (b0, b1) in zip(shares, shares[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in shares]
            assert max(sizes) - min(sizes) <= 1


def _fault_worker(rank, world, port, mode, out_q):
    """Rank 1 misbehaves according to `mode`; rank 0 runs the merge and reports what it saw.
    Every collective runs under a 3 s process-group timeout, so nothing can hang."""
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    S = 8
    if rank == 1 and mode == "raises":
        out_q.put((rank, "raised"))
        raise RuntimeError("injected failure on rank 1")  # the process exits non-zero
    if rank == 1 and mode == "late":
        time.sleep(6)  # past the others' timeout
    if rank == 1 and mode == "mismatch":
        S = 9  # a shard of another size
    t0 = time.monotonic()
    try:
        merge_across_ranks(torch.zeros(2, S, 4), torch.zeros(2, S))
        res = "no error"
    except ValueError as exc:
        res = f"ValueError: {exc}"
    except Exception as exc:  # a failed collective, not a hang
        res = f"error: {type(exc).__name__}"
    out_q.put((rank, res, time.monotonic() - t0))
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run_fault(mode):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, mode, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode is not None, "a rank hung"
    res = {}
    while not out_q.empty():
        item = out_q.get(timeout=10)
        res[item[0]] = item[1:]
    return res, [p.exitcode for p in procs]


def test_rank_that_raises_is_detected():
    res, codes = _run_fault("raises")
    assert res[1] == ("raised",) and codes[1] != 0
    assert res[0][0].startswith("error"), res[0]
    assert res[0][1] < 60


def test_rank_past_the_timeout_is_detected():
    res, _ = _run_fault("late")
    assert res[0][0].startswith("error"), res[0]
    assert res[0][1] < 60


def test_mismatched_shard_sizes_raise_on_every_rank():
    res, codes = _run_fault("mismatch")
    for rank in (0, 1):
        assert res[rank][0].startswith("ValueError"), res[rank]
        assert "differ in size" in res[rank][0]
    assert codes == [0, 0]
