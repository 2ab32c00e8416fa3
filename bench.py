"""Benchmark of the SDPA forward hot path (one JSON line on rank 0).

Workload (the config the metric is quoted on): BASELINE config 3, Llama-style prefill,
B=8, H=32, S=4096, D=128, bf16, causal, q/k/v i.i.d. N(0,1), scale 1/sqrt(128).
A step is one forward over the rank's shard of the 256 (batch, head) pairs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun (one process per GPU, NCCL only for the barrier and the
max-over-ranks of the timings). The pairs are split contiguously over the ranks with
no data-path collective (strong scaling: total work fixed).

Fields beyond the base contract:
  value     device time (CUDA events on the launching stream), inputs resident in HBM,
            an L2 flush (256 MB write) enqueued before every timed step
  e2e       same metric through tiledattention_b200.sdpa with pinned host buffers:
            every step copies q/k/v host->device and o device->host inside the timing
  roofline  tensor-bound: algorithmic FLOP per launch / average launch time vs the
            measured bf16 peak (MEASURED_PEAKS.json), traffic from the committed ncu
            summary (profiles/)
  cpu_baseline  the C oracle (float32 build, all host threads) on a bounded sample of
            the same workload (rank 0, N=1 only)
  --impl reference  times the reference's CPU path stand-in: the reference has no CPU
            implementation (its sdpa rejects non-CUDA tensors), so the arm runs the
            oracle port of its algorithm on all host threads, on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    # BASELINE config 3 (the metric's workload; default)
    "llama_prefill": {"name": "llama_prefill_b8_h32_s4096_d128_bf16_causal",
                      "B": 8, "H": 32, "S": 4096, "D": 128, "causal": True, "dtype": "bf16"},
    # BASELINE config 5 (long context)
    "long_context": {"name": "long_context_b1_h16_s65536_d128_bf16_causal",
                     "B": 1, "H": 16, "S": 65536, "D": 128, "causal": True, "dtype": "bf16"},
}
WORKLOAD = WORKLOADS["llama_prefill"]
SEED = 1234
FALLBACK_PEAK_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20


def flops(B, H, S, D, causal):
    # reference formula, benchmark-gb10/run_study.py:95-112
    return 2.0 * B * H * S * (S + 1) * D if causal else 4.0 * B * H * S * S * D


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f), "measured"
    except Exception:
        return {"bf16_tflops": FALLBACK_PEAK_TFLOPS}, "fallback"


def ncu_traffic_per_launch():
    """dram bytes (read+write) per launch of the SDPA kernel on this workload, from
    the committed ncu summary; None when no capture has been summarised yet."""
    path = os.path.join(ROOT, "profiles", "sdpa_fwd_sm100_llama_prefill.md")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) in a thread."""

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, device_index, period_s=0.02):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def make_inputs(torch, pairs, S, D, dtype, pair_start, device=None, pinned=False):
    """Seeded N(0,1) inputs for pairs [pair_start, pair_start+pairs) of the workload,
    generated per pair so every rank draws its shard independently."""
    q = torch.empty((1, pairs, S, D), dtype=dtype, pin_memory=pinned)
    k = torch.empty_like(q, pin_memory=pinned) if pinned else torch.empty_like(q)
    v = torch.empty_like(q, pin_memory=pinned) if pinned else torch.empty_like(q)
    g = torch.Generator()
    for i in range(pairs):
        g.manual_seed(SEED * 1000003 + pair_start + i)
        for t in (q, k, v):
            t[0, i].copy_(torch.randn((S, D), generator=g))
    if device is not None:
        q, k, v = (t.to(device) for t in (q, k, v))
    return q, k, v


def cpu_sample(S, D, causal, target_s):
    """Time the C oracle (float32, all host threads) on whole (b,h) pairs of the workload,
    growing the number of pairs until about target_s seconds. Returns (tflops, desc, cores)."""
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(SEED)
    cores = oracle.oracle_threads()
    pairs = 1
    while True:
        q, k, v = (rng.standard_normal((1, pairs, S, D), dtype=np.float32) for _ in range(3))
        t0 = time.perf_counter()
        oracle.sdpa_c(q, k, v, causal=causal, scale=1.0 / math.sqrt(D), precision="f32")
        dt = time.perf_counter() - t0
        if dt >= target_s * 0.5 or pairs >= 256:
            break
        pairs = min(256, max(pairs + 1, int(pairs * target_s / max(dt, 1e-3))))
    tflops = flops(1, pairs, S, D, causal) / dt / 1e12
    desc = f"{pairs} of 256 (b,h) pairs at S={S} D={D} causal={causal}, float32 C oracle, {dt:.2f} s"
    return tflops, desc, cores, dt


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOAD
    # Each step is a bounded sample; its length shrinks with the step count so that the
    # whole --steps K --warmup W run stays within about two minutes.
    default_step = min(2.0, max(0.2, 120.0 / (args.steps + 0.25 * args.warmup)))
    per_step = max(0.1, float(os.environ.get("TA_REF_STEP_S", str(default_step))))
    for _ in range(args.warmup):
        cpu_sample(wl["S"], wl["D"], wl["causal"], per_step / 4)
    vals, descs, total = [], [], 0.0
    cores = None
    for _ in range(args.steps):
        v, d, cores, dt = cpu_sample(wl["S"], wl["D"], wl["causal"], per_step)
        vals.append(v)
        descs.append(d)
        total += dt
    value = statistics.median(vals)
    line = {
        "impl": "reference",
        "metric": "sdpa_fwd_tflops",
        "value": round(value, 5),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1000 * total / max(1, args.steps), 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": wl["name"], "B": wl["B"], "H": wl["H"], "S": wl["S"],
                   "D": wl["D"], "causal": wl["causal"], "sample": descs[-1]},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores,
                         "kind": "port", "sample": descs[-1]},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation (sdpa rejects non-CUDA tensors, "
                "src/tiledattention/utils/checks.py:42-43); its cuTile GPU kernel needs cupy "
                "and tileiras (CUDA 13.1), absent from this image. This arm times the C port "
                "of its algorithm (oracle/sdpa_oracle.c, float32) on all host threads.",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama_prefill")
    ap.add_argument("--mode", choices=["bh", "split_kv"], default="bh",
                    help="bh: shard (batch, head) pairs over ranks, no collective; split_kv: "
                         "every rank takes zig-zag key slices of all pairs, NCCL log-sum-exp "
                         "merge inside the timed step (n_split=4 slices on one GPU)")
    ap.add_argument("--exchange", choices=["collective", "peer"], default="peer",
                    help="split_kv at N>1: merge the ranks' states with NCCL all-reduces "
                         "(collective) or over NVLink peer memory with this package's barrier "
                         "and merge kernels (peer)")
    ap.add_argument("--pairs", type=int, default=0,
                    help="profiling case: run only this many of the 256 (b,h) pairs")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import tiledattention_b200 as ta
    from tiledattention_b200.distributed import shard_pairs

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)

    wl = WORKLOADS[args.workload]
    B, H, S, D, causal = wl["B"], wl["H"], wl["S"], wl["D"], wl["causal"]
    dtype = torch.bfloat16
    n_pairs = args.pairs if 0 < args.pairs < B * H else B * H
    if args.mode == "split_kv":
        pair_start, pairs = 0, n_pairs  # every rank holds all pairs, splits the keys
        if world > 1:
            from tiledattention_b200.distributed import sdpa_split_kv_distributed

            def step_fn(q_, k_, v_):
                return sdpa_split_kv_distributed(q_, k_, v_, causal=causal,
                                                 exchange=args.exchange)[0]
        else:
            def step_fn(q_, k_, v_):
                return ta.sdpa_split_kv(q_, k_, v_, causal=causal, n_split=4)
    else:
        pair_start, pairs = shard_pairs(n_pairs, world, rank)

        def step_fn(q_, k_, v_):
            return ta.sdpa(q_, k_, v_, causal=causal)
    q, k, v = make_inputs(torch, pairs, S, D, dtype, pair_start, device=device)
    step_flops = flops(1, pairs, S, D, causal) / (world if args.mode == "split_kv" else 1)
    job_flops = flops(1, n_pairs, S, D, causal)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(device.index if device.index is not None else 0)
    for _ in range(args.warmup):
        flush.zero_()
        o = step_fn(q, k, v)
    torch.cuda.synchronize(device)
    ta.check_device_status(device)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler.start()
    barrier()
    torch.cuda.synchronize(device)
    for i in range(args.steps):
        flush.zero_()  # L2 flush, enqueued before the start event: not timed
        starts[i].record(stream)
        o = step_fn(q, k, v)
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    barrier()
    clocks = sampler.stop()
    ta.check_device_status(device)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(step_ms))
    avg_launch_ms = sum(step_ms) / len(step_ms)
    value = job_flops * args.steps / (total_ms / 1e3) / 1e12
    del o

    # ---- end to end through the public API, host buffers, copies inside the timing.
    # Every step copies its q, k, v host->device and its o device->host. The copies run
    # on their own streams, so step i+1's inputs travel while step i computes and step
    # i-1's output travels back (the host link is full duplex); device input buffers are
    # double-buffered and a buffer is only refilled after the step that read it finished.
    # Each copy is split in two halves (by (b,h) pairs) on two streams: two copy engines
    # move 55 GB/s host->device on a B200 where one moves 48.
    hq, hk, hv = make_inputs(torch, pairs, S, D, dtype, pair_start, pinned=True)
    bufs = [tuple(torch.empty_like(t, device=device) for t in (hq, hk, hv)) for _ in range(2)]
    ho = torch.empty_like(hq, pin_memory=True)
    e_steps = max(1, args.e2e_steps)
    h2d_streams = [torch.cuda.Stream(device) for _ in range(2)]
    d2h_streams = [torch.cuda.Stream(device) for _ in range(2)]
    ready = [[torch.cuda.Event() for _ in range(2)] for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    cut = max(1, pairs // 2)

    def halves(t):
        return (t[:, :cut], t[:, cut:]) if pairs > 1 else (t, None)

    def e2e_steps(n):
        for i in range(n):
            buf = bufs[i % 2]
            for c, cs in enumerate(h2d_streams):
                with torch.cuda.stream(cs):
                    if i >= 2:
                        cs.wait_event(done[i % 2])
                    for d_, h_ in zip(buf, (hq, hk, hv)):
                        dh, hh = halves(d_)[c], halves(h_)[c]
                        if dh is not None:
                            dh.copy_(hh, non_blocking=True)
                    ready[i % 2][c].record(cs)
            for c in range(2):
                stream.wait_event(ready[i % 2][c])
            o_ = step_fn(*buf)
            done[i % 2].record(stream)
            for c, cs in enumerate(d2h_streams):
                with torch.cuda.stream(cs):
                    cs.wait_event(done[i % 2])
                    oh, hh = halves(o_)[c], halves(ho)[c]
                    if oh is not None:
                        hh.copy_(oh, non_blocking=True)
                o_.record_stream(cs)

    e2e_steps(2)
    torch.cuda.synchronize(device)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(h2d_streams[0])
    h2d_streams[1].wait_event(e0)
    e2e_steps(e_steps)
    d2h_streams[1].wait_stream(d2h_streams[0])
    e1.record(d2h_streams[1])
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = job_flops * e_steps / (e2e_ms / 1e3) / 1e12
    elem = 2
    copies = world if args.mode == "split_kv" else 1  # split_kv: every rank copies all pairs
    h2d = 3 * n_pairs * S * D * elem * copies
    d2h = n_pairs * S * D * elem * copies

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks, peak_kind = measured_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAK_TFLOPS))
    achieved = step_flops / (avg_launch_ms / 1e3) / 1e12
    traffic = (ncu_traffic_per_launch()
               if world == 1 and args.workload == "llama_prefill" and args.mode == "bh" else None)

    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.workload == "llama_prefill":
        v_cpu, desc, cores, _ = cpu_sample(S, D, causal, float(os.environ.get("TA_CPU_SAMPLE_S", "10")))
        cpu = {"value": round(v_cpu, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": desc}

    line = {
        "metric": "sdpa_fwd_tflops",
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1), seeded per (b,h) pair",
        "config": {"workload": wl["name"] if n_pairs == B * H else f"{wl['name']}[{n_pairs} pairs]",
                   "B": B, "H": H, "S": S, "D": D, "causal": causal,
                   "pairs_per_gpu": pairs,
                   "parallelism": (f"bh-shard{world}" if args.mode == "bh" else f"split-kv{world}"),
                   **({"exchange": args.exchange} if args.mode == "split_kv" and world > 1 else {}),
                   "l2": "256 MB L2 flush enqueued before every timed step",
                   "pct_of_bf16_peak": round(100 * value / world / peak, 2)},
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e_steps,
                "path": "pinned host q,k,v -> H2D (two copy streams) -> tiledattention_b200 call -> "
                        "D2H o (two copy streams); steps pipelined, double-buffered"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} bf16_tflops (burst)",
                     "frac_of_sustained_peak": round(
                         achieved / float(peaks.get("bf16_tflops_sustained", peak)), 4),
                     "traffic": traffic},
        "cpu_baseline": cpu,
        "clocks": clocks,
        # per rank and step: bh 1 forward; split_kv on one GPU forward + combine; at N>1 two
        # zig-zag partial forwards + combine (collective) or + barrier, merge, barrier (peer)
        "gpu_launches": args.steps * world * (
            1 if args.mode == "bh" else (2 if world == 1 else (5 if args.exchange == "peer" else 3))),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
