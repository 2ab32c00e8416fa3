"""Paper-sweep harness with the reference's CSV format.

    python -m tiledattention_b200.study --out study.csv [--seq 512 1024 ...] [--dims 64 128]

Sweeps BASELINE config 2 (B=1, H=8, S in {512..8192}, D in {64, 128}, fp16/bf16,
causal/non-causal, q/k/v N(0,1), seed 1234 per config) and writes one row per
(method, config) with the columns of the reference's
benchmark-gb10/results/benchmark_results.csv:1, so results line up with its GB10 tables:

    method, baseline_name, dtype, causal, B, H, S, D, flops_forward, median_ms, p95_ms,
    throughput_tokens_per_s, tflops_per_s, approx_bw_gbps, status, status_detail

Methods: ``tiledattention`` (this package, automatic kernel choice),
``tiledattention_persistent`` / ``tiledattention_shared_kv`` (one forward kernel forced, for
dispatch sweeps; --batch/--heads widen the sweep beyond B=1, H=8) and the torch baselines
``torch_sdpa`` (auto backend) and ``torch_sdpa_math`` (math backend, on the GPU). Timing follows the
reference's time_cuda_callable (run_study.py:48-75): warm-up, then a CUDA-event pair around
every call, median and p95; the metric formulas are run_study.py:78-148. Failures are
recorded as rows with status "error" (run_study.py:338-395) instead of aborting the sweep.
"""

from __future__ import annotations

import argparse
import csv
import math
import statistics
import time

COLUMNS = [
    "method", "baseline_name", "dtype", "causal", "B", "H", "S", "D", "flops_forward",
    "median_ms", "p95_ms", "throughput_tokens_per_s", "tflops_per_s", "approx_bw_gbps",
    "status", "status_detail",
]


def attention_forward_flops(b: int, h: int, s: int, d: int, causal: bool) -> float:
    """run_study.py:95-112: causal 2*B*H*S*(S+1)*D, else 4*B*H*S^2*D."""
    return 2.0 * b * h * s * (s + 1) * d if causal else 4.0 * b * h * s * s * d


def throughput_tokens_per_s(b: int, h: int, s: int, median_ms: float) -> float:
    """run_study.py:78-92: query tokens (B*H*S) per second."""
    return b * h * s / (median_ms / 1000.0)


def approximate_bw_gbps(b: int, h: int, s: int, d: int, bytes_per_elem: int, median_ms: float) -> float:
    """run_study.py:130-148: 4*B*H*S*D*bytes moved."""
    return 4.0 * b * h * s * d * bytes_per_elem / (median_ms / 1000.0) / 1e9


def p95(values: list[float]) -> float:
    ordered = sorted(values)
    return ordered[min(len(ordered) - 1, int(math.ceil(0.95 * len(ordered))) - 1)]


def make_row(method: str, dtype_name: str, causal: bool, b: int, h: int, s: int, d: int,
             median_ms: float | None, p95_ms: float | None, status: str = "ok",
             detail: str = "") -> dict:
    flops = attention_forward_flops(b, h, s, d, causal)
    row = {
        "method": method, "baseline_name": "torch_sdpa", "dtype": dtype_name, "causal": causal,
        "B": b, "H": h, "S": s, "D": d, "flops_forward": flops,
        "median_ms": median_ms if median_ms is not None else float("nan"),
        "p95_ms": p95_ms if p95_ms is not None else float("nan"),
        "throughput_tokens_per_s": float("nan"), "tflops_per_s": float("nan"),
        "approx_bw_gbps": float("nan"), "status": status, "status_detail": detail,
    }
    if median_ms is not None and median_ms > 0:
        elem = 2 if dtype_name in ("float16", "bfloat16") else 4
        row["throughput_tokens_per_s"] = throughput_tokens_per_s(b, h, s, median_ms)
        row["tflops_per_s"] = flops / (median_ms / 1000.0) / 1e12
        row["approx_bw_gbps"] = approximate_bw_gbps(b, h, s, d, elem, median_ms)
    return row


def time_cuda_callable(torch, fn, warmup: int, iters: int, flush=None) -> tuple[float, float]:
    """Median and p95 of CUDA-event times of fn (run_study.py:48-75). `flush`: a device
    buffer larger than L2 that is rewritten before every timed call, outside the events, so
    every call starts from a cold L2 (an option beyond the reference's timing)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    timings = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        timings.append(float(start.elapsed_time(end)))
    return statistics.median(timings), p95(timings)


def run_sweep(seqs, dims, dtypes, causals, methods, warmup=5, iters=15, b=1, h=8, seed=1234,
              flush_l2=False, settle_s=0.0):
    """`settle_s` > 0: leave the GPU idle that long before timing each (shape, method), so a
    method timed right after a seconds-long heavy shape does not run in the SM-clock dip that
    follows such a load under the power cap (an option beyond the reference's timing)."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import tiledattention_b200 as ta
    from tiledattention_b200 import _native

    def forced(kind):
        def run(q, k, v, c):
            lib = _native.load_library()
            lib.ta_debug_set_kernel(kind)
            try:
                return ta.sdpa(q, k, v, causal=c)
            finally:
                lib.ta_debug_set_kernel(0)
        return run

    def torch_math(q, k, v, causal):
        with sdpa_kernel(SDPBackend.MATH):
            return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)

    impls = {
        "tiledattention": lambda q, k, v, c: ta.sdpa(q, k, v, causal=c),
        "tiledattention_persistent": forced(1),
        "tiledattention_shared_kv": forced(3),
        "torch_sdpa": lambda q, k, v, c: torch.nn.functional.scaled_dot_product_attention(
            q, k, v, is_causal=c),
        "torch_sdpa_math": torch_math,
    }
    rows = []
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush_l2 else None
    for causal in causals:
        for dtype_name in dtypes:
            dtype = getattr(torch, dtype_name)
            for s in seqs:
                for d in dims:
                    torch.manual_seed(seed)
                    q, k, v = (torch.randn(b, h, s, d, device=dev, dtype=dtype) for _ in range(3))
                    for method in methods:
                        fn = impls[method]
                        if settle_s > 0:
                            torch.cuda.synchronize()
                            time.sleep(settle_s)
                        try:
                            med, tail = time_cuda_callable(torch, lambda: fn(q, k, v, causal),
                                                           warmup, iters, flush)
                            rows.append(make_row(method, dtype_name, causal, b, h, s, d, med, tail))
                        except Exception as exc:  # recorded, like run_study.py:338-395
                            rows.append(make_row(method, dtype_name, causal, b, h, s, d, None,
                                                 None, "error", f"{type(exc).__name__}: {exc}"))
                    del q, k, v
    return rows


def write_csv(rows, path: str) -> None:
    with open(path, "w", newline="") as f:
        writer = csv.DictWriter(f, fieldnames=COLUMNS)
        writer.writeheader()
        writer.writerows(rows)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="study.csv")
    ap.add_argument("--seq", type=int, nargs="+", default=[512, 1024, 2048, 4096, 8192])
    ap.add_argument("--dims", type=int, nargs="+", default=[64, 128])
    ap.add_argument("--dtypes", nargs="+", default=["float16", "bfloat16"])
    ap.add_argument("--causal", nargs="+", default=["False", "True"])
    ap.add_argument("--methods", nargs="+", default=["tiledattention", "torch_sdpa", "torch_sdpa_math"])
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=15)
    ap.add_argument("--batch", type=int, nargs="+", default=[1])
    ap.add_argument("--heads", type=int, nargs="+", default=[8])
    ap.add_argument("--flush-l2", action="store_true",
                    help="rewrite a 256 MB buffer before every timed call (cold L2)")
    ap.add_argument("--settle-s", type=float, default=0.0,
                    help="idle seconds before timing each (shape, method); 0 as the reference")
    args = ap.parse_args(argv)
    rows = []
    for b in args.batch:
        for h in args.heads:
            rows += run_sweep(args.seq, args.dims, args.dtypes, [c == "True" for c in args.causal],
                              args.methods, args.warmup, args.iters, b=b, h=h,
                              flush_l2=args.flush_l2, settle_s=args.settle_s)
    write_csv(rows, args.out)
    print(f"wrote {len(rows)} rows to {args.out}")


if __name__ == "__main__":
    main()
