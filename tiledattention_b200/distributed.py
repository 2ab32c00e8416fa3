"""Multi-GPU orchestration for the SDPA forward (one process per GPU, torch.distributed).

Two ways to spread one attention forward over a group of ranks (the reference has no
multi-GPU code; both are new):

* (batch, head) sharding — pairs are independent, so each rank takes a contiguous range
  of the B*H pairs and no collective is needed (``shard_pairs``).
* split-KV — every rank holds q, k, v for all heads and attends all query rows to its own
  key slices, chosen zig-zag so that causal work is balanced (``zigzag_key_ranges``); the
  per-rank (o, lse) states are merged with a log-sum-exp combine: an all-reduce(MAX) of
  lse, local weights w = exp(lse - lse_max), then one all-reduce(SUM) of [w*o | w]
  (``merge_across_ranks``). The merge works on any device / backend (NCCL on GPUs,
  gloo on CPU for tests).
"""

from __future__ import annotations

import math

KEY_TILE = 128


def shard_pairs(n_pairs: int, world: int, rank: int) -> tuple[int, int]:
    """(first pair, pair count) of `rank` when n_pairs are split contiguously."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid world / rank")
    base, rem = divmod(n_pairs, world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def zigzag_key_ranges(seq_len: int, world: int, rank: int, tile: int = KEY_TILE):
    """Key ranges of `rank`: the keys are cut into 2*world tile-aligned chunks and rank r
    takes chunks r and 2*world-1-r, so every rank gets one early (expensive under a causal
    mask) and one late (cheap) chunk. Returns a list of (begin, end), empty ones dropped."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid world / rank")
    n_chunks = 2 * world
    chunk = max(tile, math.ceil(math.ceil(seq_len / n_chunks) / tile) * tile)
    out = []
    for c in (rank, n_chunks - 1 - rank):
        lo, hi = min(seq_len, c * chunk), min(seq_len, (c + 1) * chunk)
        if hi > lo:
            out.append((lo, hi))
    return sorted(out)


def lse_merge(o_parts, lse_parts):
    """Merge partial states along dim 0: o_parts [n, ..., D] fp32, lse_parts [n, ...].
    Returns (o, lse) with o = sum_i exp(lse_i - lse) o_i, lse = log sum_i exp(lse_i);
    rows whose partials are all -inf give o = 0, lse = -inf."""
    import torch

    m = lse_parts.max(dim=0).values
    safe_m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse_parts - safe_m)  # exp(-inf) = 0 for empty partials
    den = w.sum(dim=0)
    num = (o_parts * w.unsqueeze(-1)).sum(dim=0)
    o = torch.where(den.unsqueeze(-1) > 0, num / den.clamp_min(1e-30).unsqueeze(-1),
                    torch.zeros_like(num))
    lse = torch.where(den > 0, safe_m + torch.log(den.clamp_min(1e-30)),
                      torch.full_like(den, -math.inf))
    return o, lse


def merge_across_ranks(o_part, lse_part, group=None):
    """Collective log-sum-exp merge: every rank passes its fp32 partial (o_part [..., D],
    lse_part [...]) and gets the merged (o, lse) of all ranks. Two collectives: an
    all-reduce(MAX) of lse and an all-reduce(SUM) of [w*o | w]."""
    import torch
    import torch.distributed as dist

    lse_max = lse_part.clone()
    dist.all_reduce(lse_max, op=dist.ReduceOp.MAX, group=group)
    safe_m = torch.where(torch.isfinite(lse_max), lse_max, torch.zeros_like(lse_max))
    w = torch.exp(lse_part - safe_m)
    buf = torch.cat([o_part * w.unsqueeze(-1), w.unsqueeze(-1)], dim=-1)
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    num, den = buf[..., :-1], buf[..., -1]
    o = torch.where(den.unsqueeze(-1) > 0, num / den.clamp_min(1e-30).unsqueeze(-1),
                    torch.zeros_like(num))
    lse = torch.where(den > 0, safe_m + torch.log(den.clamp_min(1e-30)),
                      torch.full_like(den, -math.inf))
    return o, lse


def sdpa_split_kv_distributed(q, k, v, *, causal: bool = False, scale: float | None = None,
                              group=None):
    """Split-KV SDPA across the ranks of `group` (one GPU each): this rank attends all
    query rows of q to its zig-zag key slices with the sm_100a kernel, merges its slices
    on the GPU, and the ranks merge their states with merge_across_ranks. Every rank
    returns the full output (dtype of q) and the fp32 lse."""
    import torch
    import torch.distributed as dist

    from .launch import run_lse_combine
    from .sdpa import sdpa_partial

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    seq_len = int(q.shape[2])
    parts_o, parts_l = [], []
    for lo, hi in zigzag_key_ranges(seq_len, world, rank):
        o_p, l_p = sdpa_partial(q, k, v, causal=causal, scale=scale, kv_begin=lo, kv_end=hi)
        parts_o.append(o_p)
        parts_l.append(l_p)
    if parts_o:
        o_local, lse_local = run_lse_combine(torch.cat(parts_o).contiguous(),
                                             torch.cat(parts_l).contiguous(),
                                             out_dtype=torch.float32, return_lse=True)
        o_local = o_local[..., : q.shape[-1]]
    else:
        o_local = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        lse_local = torch.full(q.shape[:3], -math.inf, dtype=torch.float32, device=q.device)
    o, lse = merge_across_ranks(o_local.contiguous(), lse_local, group=group)
    return o.to(q.dtype), lse
