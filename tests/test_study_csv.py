"""The study harness writes the reference's CSV format
(benchmark-gb10/results/benchmark_results.csv:1) and computes its metrics with the
reference's formulas; the known answers below are the reference's own published row 2
(tiledattention, float16, non-causal, B1 H8 S512 D64, median 0.035328 ms)."""

import csv

import pytest

from tiledattention_b200 import study

REFERENCE_HEADER = ("method,baseline_name,dtype,causal,B,H,S,D,flops_forward,median_ms,p95_ms,"
                    "throughput_tokens_per_s,tflops_per_s,approx_bw_gbps,status,status_detail")


def test_columns_match_reference_header():
    assert ",".join(study.COLUMNS) == REFERENCE_HEADER


def test_metrics_match_reference_row():
    row = study.make_row("tiledattention", "float16", False, 1, 8, 512, 64,
                         0.03532800078392029, 0.04794240221381187)
    assert row["flops_forward"] == 536870912.0
    assert row["throughput_tokens_per_s"] == pytest.approx(115942026.41278003, rel=1e-12)
    assert row["tflops_per_s"] == pytest.approx(15.196753285975904, rel=1e-12)
    assert row["approx_bw_gbps"] == pytest.approx(59.36231752334338, rel=1e-12)


def test_error_rows_and_csv_roundtrip(tmp_path):
    rows = [study.make_row("tiledattention", "bfloat16", True, 1, 8, 4096, 128, 0.5, 0.6),
            study.make_row("torch_sdpa_math", "bfloat16", True, 1, 8, 8192, 128, None, None,
                           "error", "OutOfMemoryError: ...")]
    path = tmp_path / "s.csv"
    study.write_csv(rows, str(path))
    lines = path.read_text().splitlines()
    assert lines[0] == REFERENCE_HEADER
    back = list(csv.DictReader(open(path)))
    assert back[0]["status"] == "ok" and back[1]["status"] == "error"
    assert float(back[0]["flops_forward"]) == 2 * 8 * 4096 * 4097 * 128


def test_settle_option_reaches_the_sweep(tmp_path, monkeypatch):
    seen = {}

    def fake_sweep(*args, **kwargs):
        seen.update(kwargs)
        return []

    monkeypatch.setattr(study, "run_sweep", fake_sweep)
    out = tmp_path / "s.csv"
    study.main(["--out", str(out), "--settle-s", "0.5", "--seq", "512"])
    assert seen["settle_s"] == 0.5
    assert out.read_text().startswith(REFERENCE_HEADER)
    seen.clear()
    study.main(["--out", str(out), "--seq", "512"])
    assert seen["settle_s"] == 0.0  # default: the reference harness's timing
