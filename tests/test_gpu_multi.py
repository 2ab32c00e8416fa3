"""Split-KV across GPUs: two ranks (one process per GPU, NCCL) attend all query rows to
their zig-zag key slices with the sm_100a kernel and merge by log-sum-exp
(tiledattention_b200.distributed.sdpa_split_kv_distributed), either with all-reduces or over
NVLink peer memory with the package's own barrier and merge kernels; the result is compared
with the float64 oracle on sampled rows. NVLS is disabled for this test. Skipped with fewer
than two GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out_q, exchange):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    import tiledattention_b200 as ta
    from tiledattention_b200.distributed import sdpa_split_kv_distributed

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        g = torch.Generator().manual_seed(7)
        S, D = 8192, 128
        q, k, v = (torch.randn(1, 2, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        if exchange == "peer":
            # Warm the exchange (and its alternating state sets) with other inputs first.
            for i in range(3):
                sdpa_split_kv_distributed(qd * (i + 2), kd, vd, causal=True, exchange="peer")
        o, lse = sdpa_split_kv_distributed(qd, kd, vd, causal=True, exchange=exchange)
        ta.check_device_status(dev)
        if exchange == "peer":
            o_c, lse_c = sdpa_split_kv_distributed(qd, kd, vd, causal=True)
            assert (o.float() - o_c.float()).abs().max().item() <= 2.0 ** -7
            assert (lse - lse_c).abs().max().item() <= 1e-4
            from tiledattention_b200.distributed import peer_exchange_for, row_share

            ex = peer_exchange_for(qd, D)
            o_part, lse_part, (b0, b1) = ex.forward(qd, kd, vd, causal=True, scale=D ** -0.5,
                                                     gather=False)
            assert (b0, b1) == row_share(S, world, rank)
            assert torch.equal(o_part, o[:, :, b0:b1])
            assert torch.equal(lse_part, lse[:, :, b0:b1])
            ta.check_device_status(dev)
        from oracle import oracle

        rows = (S - 96, S)
        ref = torch.from_numpy(oracle.sdpa_c(q, k, v, causal=True, scale=D ** -0.5, rows=rows))
        got = o.float().cpu()[:, :, rows[0]:rows[1]]
        ref = ref[:, :, rows[0]:rows[1]]
        bound = 1e-2 + 2.0 ** -8 * ref.abs()
        out_q.put((rank, float(((got - ref).abs() - bound).max()), float((got - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["collective", "peer"])
def test_split_kv_two_gpus(exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out_q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for _ in range(2):
        rank, worst, err = out_q.get(timeout=10)
        assert worst <= 0, (rank, err)
