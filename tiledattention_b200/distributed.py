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

On GPUs the exchange can instead run over NVLink peer memory with this package's own
kernels (``PeerExchange``): the per-rank states are written into a buffer every rank has
mapped (torch symmetric memory), a bounded device barrier (ta_peer_barrier) orders them,
and one merge kernel per rank reads its share of query rows from every peer and writes the
merged rows — to itself (a reduce-scatter by rows) or to every rank (the all-gather fused
into the same pass). No collective library is in that data path.
"""

from __future__ import annotations

import ctypes
import math
import os

KEY_TILE = 128
SLICES_PER_RANK = 2  # zig-zag: every rank owns two key ranges


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


def merge_across_ranks(o_part, lse_part, group=None, validate: bool | None = None):
    """Collective log-sum-exp merge: every rank passes its fp32 partial (o_part [..., D],
    lse_part [...]) and gets the merged (o, lse) of all ranks. Two collectives: an
    all-reduce(MAX) of lse and an all-reduce(SUM) of [w*o | w].

    validate: first agree on the partials' sizes with one small all-reduce and raise
    ValueError on every rank if they differ (mismatched shards would otherwise make the
    collectives fail obscurely or combine unrelated rows). Default: on for host tensors; for
    device tensors it costs a host synchronisation, so it is opt-in there."""
    import torch
    import torch.distributed as dist

    if validate is None:
        validate = lse_part.device.type == "cpu"
    if validate:
        n, d = lse_part.numel(), int(o_part.shape[-1])
        sizes = torch.tensor([n, -n, d, -d, o_part.numel(), -o_part.numel()], dtype=torch.int64,
                             device=lse_part.device)
        dist.all_reduce(sizes, op=dist.ReduceOp.MAX, group=group)
        lo_hi = sizes.tolist()
        if (lo_hi[0] != -lo_hi[1] or lo_hi[2] != -lo_hi[3] or lo_hi[4] != -lo_hi[5]
                or o_part.numel() != n * d):
            raise ValueError("merge_across_ranks: the ranks' partial states differ in size "
                             f"(this rank: lse {tuple(lse_part.shape)}, o "
                             f"{tuple(o_part.shape)})")

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


def row_share(seq_len: int, world: int, rank: int) -> tuple[int, int]:
    """Query rows [begin, end) whose merge `rank` performs in the peer exchange."""
    base, extra = divmod(seq_len, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerExchange:
    """Split-KV state exchange over NVLink peer memory for one (shape, dtype, group).

    Holds one symmetric-memory allocation per rank, mapped by every peer, laid out as
        [flags: TA_MAX_PEERS uint32 | pad to 256 B]
        2 x [o_state fp32 [2][B*H][S][Dk] | lse_state fp32 [2][B*H*S]
             | out (dtype) [B*H][S][Dk] | lse_out fp32 [B*H*S]]
    The two state sets alternate between calls, so a rank never overwrites a state a peer
    may still be reading (the barrier of the next call orders that). Every rank must call
    ``forward`` the same number of times, in the same order.
    """

    def __init__(self, shape, dtype, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from . import _native

        self.torch = torch
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > _native.TA_MAX_PEERS:
            raise ValueError(f"peer exchange serves at most {_native.TA_MAX_PEERS} ranks")
        batch, heads, seq_len, kdim = (int(x) for x in shape)
        self.shape, self.dtype, self.device = (batch, heads, seq_len, kdim), dtype, device
        rows = batch * heads * seq_len
        elem = torch.empty((), dtype=dtype).element_size()
        self.off = {}
        cur = 256
        for st in range(2):
            for name, nbytes in (("o_state", SLICES_PER_RANK * rows * kdim * 4),
                                 ("lse_state", SLICES_PER_RANK * rows * 4),
                                 ("out", rows * kdim * elem), ("lse_out", rows * 4)):
                self.off[(name, st)] = cur
                cur = _align(cur + nbytes)
        self.nbytes = cur
        try:
            symm_mem.enable_symm_mem_for_group(self.group.group_name)
        except Exception:  # newer torch: rendezvous needs no enabling
            pass
        self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.peer_base = [int(p) for p in self.handle.buffer_ptrs]
        self.buf[:256].zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)
        self.epoch = 0
        self.calls = 0
        self.timeout_ns = int(float(os.getenv("TILEDATTN_PEER_TIMEOUT_MS", "10000")) * 1e6)
        self._flag_ptrs = (ctypes.c_void_p * self.world)(*self.peer_base)

    def _view(self, name: str, st: int, dtype, shape):
        start = self.off[(name, st)]
        count = math.prod(shape)
        nbytes = count * self.torch.empty((), dtype=dtype).element_size()
        return self.buf[start:start + nbytes].view(dtype).view(shape)

    def _barrier(self, lib, status, stream):
        from .launch import _raise_for

        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        rc = lib.ta_peer_barrier(ctypes.addressof(self._flag_ptrs), self.world, self.rank,
                                 self.epoch, self.timeout_ns, status.data_ptr(), stream)
        if rc != 0:
            _raise_for(lib, rc)

    def forward(self, q, k, v, *, causal: bool, scale: float, gather: bool = True):
        """Split-KV forward of this rank's zig-zag key slices, then the peer exchange.

        gather=True: every rank returns the full o [B,H,S,D] (dtype of q) and lse [B,H,S].
        gather=False: this rank returns only its merged query rows o [B,H,rows,D] and lse
        [B,H,rows], plus (begin, end) of those rows (row_share).
        """
        from . import _native, _runtime
        from .launch import _dtype_code, _raise_for, _status_word, run_sdpa_partial

        torch = self.torch
        lib = _runtime.get_native_library()
        batch, heads, seq_len, kdim = self.shape
        head_dim = int(q.shape[-1])
        st = self.calls % 2
        self.calls += 1
        o_state = self._view("o_state", st, torch.float32,
                             (SLICES_PER_RANK, batch, heads, seq_len, kdim))
        lse_state = self._view("lse_state", st, torch.float32,
                               (SLICES_PER_RANK, batch, heads, seq_len))
        ranges = list(zigzag_key_ranges(seq_len, self.world, self.rank))
        for j in range(SLICES_PER_RANK):
            if j < len(ranges):
                lo, hi = ranges[j]
                run_sdpa_partial(q, k, v, causal=causal, scale=scale, kv_begin=lo, kv_end=hi,
                                 out=(o_state[j:j + 1], lse_state[j:j + 1]))
            else:
                lse_state[j].fill_(-math.inf)
        with torch.cuda.device(q.device):
            stream = torch.cuda.current_stream(q.device).cuda_stream
            status = _status_word(torch, q.device)
            self._barrier(lib, status, stream)
            o_src, l_src = [], []
            for base in self.peer_base:
                for j in range(SLICES_PER_RANK):
                    o_src.append(base + self.off[("o_state", st)] + j * batch * heads * seq_len * kdim * 4)
                    l_src.append(base + self.off[("lse_state", st)] + j * batch * heads * seq_len * 4)
            s_begin, s_end = row_share(seq_len, self.world, self.rank)
            o_src_arr = (ctypes.c_void_p * len(o_src))(*o_src)
            l_src_arr = (ctypes.c_void_p * len(l_src))(*l_src)
            code = _dtype_code(torch, q.dtype)
            if gather:
                dsts = [b + self.off[("out", st)] for b in self.peer_base]
                ldsts = [b + self.off[("lse_out", st)] for b in self.peer_base]
                strides = (heads * seq_len * kdim, seq_len * kdim, kdim, 1)
                out_rows, row_base = seq_len, 0
                result = None
            else:
                rows = s_end - s_begin
                result = torch.empty((batch, heads, rows, kdim), dtype=q.dtype, device=q.device)
                lse_res = torch.empty((batch, heads, rows), dtype=torch.float32, device=q.device)
                dsts, ldsts = [result.data_ptr()], [lse_res.data_ptr()]
                strides = tuple(result.stride())
                out_rows, row_base = rows, s_begin
            dst_arr = (ctypes.c_void_p * len(dsts))(*dsts)
            ldst_arr = (ctypes.c_void_p * len(ldsts))(*ldsts)
            if s_end > s_begin:
                rc = lib.ta_lse_merge_peers(
                    ctypes.addressof(o_src_arr), ctypes.addressof(l_src_arr), len(o_src),
                    batch, heads, seq_len, kdim, s_begin, s_end, ctypes.addressof(dst_arr),
                    ctypes.addressof(ldst_arr), len(dsts), _native.strides4(strides), out_rows,
                    row_base, code, status.data_ptr(), stream)
                if rc != 0:
                    _raise_for(lib, rc)
            if not gather:
                return result[..., :head_dim], lse_res, (s_begin, s_end)
            self._barrier(lib, status, stream)
            o = self._view("out", st, q.dtype, (batch, heads, seq_len, kdim))[..., :head_dim].clone()
            lse = self._view("lse_out", st, torch.float32, (batch, heads, seq_len)).clone()
        return o, lse


_exchanges: dict = {}


def peer_exchange_for(q, kdim: int, group=None) -> PeerExchange:
    """The cached PeerExchange for q's shape / dtype / device and `group`."""
    key = (tuple(q.shape[:3]), kdim, q.dtype, q.device.index, id(group))
    ex = _exchanges.get(key)
    if ex is None:
        ex = PeerExchange((*q.shape[:3], kdim), q.dtype, q.device, group)
        _exchanges[key] = ex
    return ex


def sdpa_split_kv_distributed(q, k, v, *, causal: bool = False, scale: float | None = None,
                              group=None, exchange: str = "collective"):
    """Split-KV SDPA across the ranks of `group` (one GPU each): this rank attends all
    query rows of q to its zig-zag key slices with the sm_100a kernel, and the ranks merge
    their states. Every rank returns the full output (dtype of q) and the fp32 lse.

    exchange="collective": the rank merges its slices on the GPU, then merge_across_ranks
    (all-reduces; any backend). exchange="peer": PeerExchange over NVLink peer memory
    (CUDA tensors, every rank's GPU reachable by load/store from every other)."""
    import torch
    import torch.distributed as dist

    from .launch import run_lse_combine, state_head_dim
    from .sdpa import _prepare, sdpa_partial

    if exchange == "peer":
        resolved = _prepare(q, k, v, causal, scale)
        ex = peer_exchange_for(q, state_head_dim(int(q.shape[-1])), group)
        return ex.forward(q, k, v, causal=causal, scale=resolved, gather=True)
    if exchange != "collective":
        raise ValueError("exchange must be 'collective' or 'peer'")

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
