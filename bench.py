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
  max_abs_err  the last timed step's output checked, after the timed region, against the
            float64 oracle on sampled query-row blocks of sampled (b,h) pairs (max over
            ranks), with the tolerance it must meet
  sustained a seconds-long loop of the same step after the timed region, with its own
            clock record, judged against the sustained bf16 peak (bf16_tflops_sustained)
  ranks     (N > 1) each rank's step-time median / min / max, its kernel time, SM clock
            median and GPU utilisation during the timed region, and how many were busy
  context   torch's own GPU SDPA (scaled_dot_product_attention, default backend choice)
            on the same inputs, timed the same way (N = 1): a same-box comparison only
  cpu_baseline  the reference's CPU path as north_star names it: torch SDPA math backend
            in float32 on all host threads, on a bounded sample of the same workload
            (rank 0, N=1 only); the C oracle port's rate on the same sample is reported
            beside it ("port")
  --impl reference  times that same CPU path (torch SDPA math, float32, all host threads):
            the reference has no CPU implementation of its own (its sdpa rejects non-CUDA
            tensors) and its cuTile GPU kernel cannot run on this image.
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
# The L2 statement of the timing contract; part of both arms' `config`, which describes the
# workload only (run details such as the sharding go to `run`), so the two arms' configs agree.
L2_NOTE = ("inputs larger than the 126 MB L2 (q, k, v 805 MB at config 3) and a 256 MB L2 "
           "flush enqueued before every timed GPU step")


def workload_config(wl, n_pairs=None):
    name = wl["name"] if not n_pairs or n_pairs == wl["B"] * wl["H"] else f"{wl['name']}[{n_pairs} pairs]"
    return {"workload": name, "B": wl["B"], "H": wl["H"], "S": wl["S"], "D": wl["D"],
            "causal": wl["causal"], "l2": L2_NOTE}


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


def _nvml_handle(torch, device):
    """NVML handle of a torch CUDA device, matched by PCI address (CUDA_VISIBLE_DEVICES may
    renumber devices), falling back to the same index; (None, None) without NVML."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(device)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
    except Exception:
        return None, None


class ClockSampler:
    """Samples SM clock, GPU utilisation and throttle reasons through NVML (read-only) in a
    thread."""

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, torch, device, period_s=0.02):
        self.samples = []
        self.util = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self._nvml, self._h = _nvml_handle(torch, device)
        if self._nvml is not None:
            try:
                self.max_mhz = self._nvml.nvmlDeviceGetMaxClockInfo(self._h, self._nvml.NVML_CLOCK_SM)
            except Exception:
                self._nvml = None

    def _sample(self):
        nv = self._nvml
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
            self.util.append(nv.nvmlDeviceGetUtilizationRates(self._h).gpu)
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            for name, bit in self.REASONS.items():
                if mask & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            if len(self.samples) < 2:  # a run shorter than the period: one more sample
                self._sample()
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }

    def util_max(self):
        return max(self.util) if self.util else None


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


def _cpu_pairs(pairs, S, D):
    import numpy as np

    rng = np.random.default_rng(SEED)
    return [rng.standard_normal((1, pairs, S, D), dtype=np.float32) for _ in range(3)]


def cpu_sample_torch_math(S, D, causal, target_s):
    """The reference's CPU path as its benchmarks define it (torch SDPA, math backend,
    float32; benchmark-gb10/run_study.py:249-271) on all host threads, over whole (b,h)
    pairs of the workload, growing the number of pairs until about target_s seconds.
    Returns (tflops, desc, cores, seconds, pairs)."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    pairs = 1
    while True:
        q, k, v = (torch.from_numpy(a) for a in _cpu_pairs(pairs, S, D))
        t0 = time.perf_counter()
        with sdpa_kernel(SDPBackend.MATH):
            for i in range(pairs):  # one pair at a time: the S x S score matrix stays small
                torch.nn.functional.scaled_dot_product_attention(
                    q[:, i:i + 1], k[:, i:i + 1], v[:, i:i + 1], is_causal=causal,
                    scale=1.0 / math.sqrt(D))
        dt = time.perf_counter() - t0
        if dt >= target_s * 0.5 or pairs >= 256:
            break
        pairs = min(256, max(pairs + 1, int(pairs * target_s / max(dt, 1e-3))))
    tflops = flops(1, pairs, S, D, causal) / dt / 1e12
    desc = (f"{pairs} of 256 (b,h) pairs at S={S} D={D} causal={causal}, torch "
            f"{torch.__version__} scaled_dot_product_attention math backend, float32, "
            f"{cores} threads, {dt:.2f} s")
    return tflops, desc, cores, dt, pairs


def cpu_sample_port(S, D, causal, pairs):
    """The float32 C oracle port (all host threads) on the same pairs. Returns
    (tflops, desc, cores)."""
    from oracle import oracle

    q, k, v = _cpu_pairs(pairs, S, D)
    cores = oracle.oracle_threads()
    t0 = time.perf_counter()
    oracle.sdpa_c(q, k, v, causal=causal, scale=1.0 / math.sqrt(D), precision="f32")
    dt = time.perf_counter() - t0
    return (flops(1, pairs, S, D, causal) / dt / 1e12,
            f"{pairs} (b,h) pairs, float32 C oracle port, {cores} threads, {dt:.2f} s", cores)


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOAD
    # Each step is a bounded sample; its length shrinks with the step count so that the
    # whole --steps K --warmup W run stays within about two minutes.
    default_step = min(2.0, max(0.2, 120.0 / (args.steps + 0.25 * args.warmup)))
    per_step = max(0.1, float(os.environ.get("TA_REF_STEP_S", str(default_step))))
    for _ in range(args.warmup):
        cpu_sample_torch_math(wl["S"], wl["D"], wl["causal"], per_step / 4)
    vals, descs, total = [], [], 0.0
    cores = None
    for _ in range(args.steps):
        v, d, cores, dt, _ = cpu_sample_torch_math(wl["S"], wl["D"], wl["causal"], per_step)
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
        "config": workload_config(wl),
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores,
                         "kind": "reference", "sample": descs[-1], "cpu": _cpu_model()},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's CPU path as north_star defines it: torch SDPA math backend in "
                "float32 on all host threads (the reference's own sdpa rejects non-CUDA tensors, "
                "src/tiledattention/utils/checks.py:42-43, and its cuTile GPU kernel needs cupy "
                "and tileiras (CUDA 13.1), absent from this image).",
    }
    print(json.dumps(line), flush=True)


def self_check(torch, o, q, k, v, causal, world):
    """Max-abs error of the step's output against the float64 oracle on the first and last
    128-row block of the first, middle and last (b,h) pair of this rank's shard (outside the
    timed region). Returns (max error over ranks, description)."""
    import numpy as np

    from oracle import oracle

    pairs, S, D = q.shape[1], q.shape[2], q.shape[3]
    idx = sorted({0, pairs // 2, pairs - 1})
    blocks = [(0, min(S, 128)), (max(0, S - 128), S)]
    qs, ks, vs, os_ = (t[:, idx].float().cpu() for t in (q, k, v, o))
    err = 0.0
    for r0, r1 in blocks:
        ref = oracle.sdpa_c(qs, ks, vs, causal=causal, scale=1.0 / math.sqrt(D), rows=(r0, r1))
        err = max(err, float(np.abs(os_[:, :, r0:r1].numpy() - ref[:, :, r0:r1]).max()))
    return err, f"rows {blocks} of pairs {idx} of each rank's shard vs the float64 oracle"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sustained-s", type=float, default=4.0,
                    help="length of the sustained-regime loop after the timed region (0: skip)")
    ap.add_argument("--no-context", action="store_true",
                    help="skip timing torch's own GPU SDPA on the same inputs")
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
                    help="profiling case: run only this many of the (b,h) pairs")
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

    def timed_loop(n, fn):
        """n steps, each after an (untimed) L2 flush; per-step device times in ms. A ~50 ms
        device-side sleep is enqueued first (outside every timed window) so that the host has
        enqueued the steps before the GPU reaches them: otherwise a host-side hiccup while the
        first steps are enqueued leaves the GPU idle between a step's start event and its kernel
        (seen as one 2 ms step of 0.14 ms ones at N=8)."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        out = None
        torch.cuda._sleep(int(50e-3 * 2.0e9))  # ~50 ms at up to 2 GHz
        for i in range(n):
            flush.zero_()  # L2 flush, enqueued before the start event: not timed
            starts[i].record(stream)
            out = fn(q, k, v)
            ends[i].record(stream)
        torch.cuda.synchronize(device)
        return [s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)], out

    # The process group's first collectives set up NCCL communicators (tens of ms); run them
    # here so that no timed step waits for that set-up.
    barrier()
    max_over_ranks(0.0)
    torch.cuda.synchronize(device)
    sampler = ClockSampler(torch, device)
    for _ in range(args.warmup):
        flush.zero_()
        o = step_fn(q, k, v)
    torch.cuda.synchronize(device)
    ta.check_device_status(device)

    sampler.start()
    barrier()
    torch.cuda.synchronize(device)
    step_ms, o = timed_loop(args.steps, step_fn)
    barrier()
    clocks = sampler.stop()
    ta.check_device_status(device)
    total_ms = max_over_ranks(sum(step_ms))
    avg_launch_ms = sum(step_ms) / len(step_ms)
    value = job_flops * args.steps / (total_ms / 1e3) / 1e12

    # ---- correctness of what was timed (outside the timed region)
    tol = 1e-2  # bfloat16 max-abs bound of north_star
    err = max_over_ranks(self_check(torch, o, q, k, v, causal, world)[0])
    check_desc = self_check.__doc__.split("(")[0].strip()
    del o

    # ---- per-rank record (N > 1): where the time goes on each GPU
    ranks = None
    if world > 1:
        mine = {"rank": rank, "pairs": pairs,
                "step_ms_median": round(statistics.median(step_ms), 4),
                "step_ms_min": round(min(step_ms), 4), "step_ms_max": round(max(step_ms), 4),
                "step_max_index": int(max(range(len(step_ms)), key=lambda i: step_ms[i])),
                "kernel_ms_total": round(sum(step_ms), 4),
                "sm_mhz": clocks["sm_mhz"], "reasons": clocks["reasons"]}
        ranks = {"mine": mine}

    # ---- sustained regime: several seconds of the same step, with its own clock record
    sustained = None
    if args.sustained_s > 0:
        n_sus = max(200, int(args.sustained_s * 1000 / max(avg_launch_ms + 0.05, 1e-3)))
        sus_sampler = ClockSampler(torch, device)
        sus_sampler.start()
        barrier()
        sus_ms, o = timed_loop(n_sus, step_fn)
        barrier()
        sus_clocks = sus_sampler.stop()
        del o
        sus_total = max_over_ranks(sum(sus_ms))
        sus_util = sus_sampler.util_max()
        sus_value = job_flops * n_sus / (sus_total / 1e3) / 1e12
        sustained = {"value": round(sus_value, 2), "steps": n_sus,
                     "seconds": round(sus_total / 1e3, 2), "clocks": sus_clocks}
        if ranks is not None:
            ranks["mine"]["gpu_util_max"] = sus_util

    # ---- per-rank record gathered on rank 0 (after the sustained loop, whose seconds of work
    # give NVML's utilisation counter, averaged over its own window, time to see each GPU busy)
    if ranks is not None:
        gathered = [None] * world
        dist.all_gather_object(gathered, ranks["mine"])
        ranks = {"per_rank": gathered,
                 "gpus_busy": sum(1 for r in gathered if (r.get("gpu_util_max") or 0) > 0),
                 "step_ms_spread": round(max(r["step_ms_median"] for r in gathered) -
                                         min(r["step_ms_median"] for r in gathered), 4)}

    # ---- same-box context: torch's own GPU SDPA on the same inputs, timed the same way
    context = None
    if world == 1 and not args.no_context and args.mode == "bh":
        try:
            def torch_sdpa(q_, k_, v_):
                return torch.nn.functional.scaled_dot_product_attention(q_, k_, v_, is_causal=causal)

            for _ in range(3):
                torch_sdpa(q, k, v)
            t_ms, o = timed_loop(max(5, min(args.steps, 50)), torch_sdpa)
            del o
            context = {"torch_sdpa_gpu_tflops": round(step_flops * len(t_ms) / (sum(t_ms) / 1e3) / 1e12, 2),
                       "what": f"torch {torch.__version__} F.scaled_dot_product_attention "
                               "(default backend choice) on the same inputs, same flush/timing"}
        except Exception as exc:  # context only: never fails the bench
            context = {"error": repr(exc)[:200]}

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
    peak_sus = float(peaks.get("bf16_tflops_sustained", peak))
    achieved = step_flops / (avg_launch_ms / 1e3) / 1e12
    traffic = (ncu_traffic_per_launch()
               if world == 1 and args.workload == "llama_prefill" and args.mode == "bh" else None)
    if sustained is not None:
        sustained["frac_of_sustained_peak"] = round(sustained["value"] / world / peak_sus, 4)
        sustained["peak_sustained"] = peak_sus

    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.workload == "llama_prefill":
        v_cpu, desc, cores, _, cpu_pairs = cpu_sample_torch_math(
            S, D, causal, float(os.environ.get("TA_CPU_SAMPLE_S", "10")))
        v_port, desc_port, cores_port = cpu_sample_port(S, D, causal, cpu_pairs)
        cpu = {"value": round(v_cpu, 5), "unit": "TFLOP/s", "cores": cores, "kind": "reference",
               "sample": desc, "cpu": _cpu_model(),
               "port": {"value": round(v_port, 5), "cores": cores_port, "sample": desc_port}}

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
        "config": workload_config(wl, n_pairs),
        "run": {"pairs_per_gpu": pairs,
                "parallelism": (f"bh-shard{world}" if args.mode == "bh" else f"split-kv{world}"),
                **({"exchange": args.exchange} if args.mode == "split_kv" and world > 1 else {}),
                "pct_of_bf16_peak_per_gpu": round(100 * value / world / peak, 2)},
        "max_abs_err": {"value": err, "tol": tol, "pass": bool(err <= tol), "what": check_desc},
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e_steps,
                "path": "pinned host q,k,v -> H2D (two copy streams) -> tiledattention_b200 call -> "
                        "D2H o (two copy streams); steps pipelined, double-buffered"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} bf16_tflops (burst)",
                     "frac_of_sustained_peak": round(achieved / peak_sus, 4),
                     "traffic": traffic},
        "sustained": sustained,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "ranks": ranks,
        "context": context,
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
