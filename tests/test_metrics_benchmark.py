"""Metric-window latency harness on CPU: one-process and gloo-merged AUC / GAUC / calibration agree,
sample counts are checked, and the timing summaries have the reference harness's fields."""
import json

import pytest

from flare_b200.benchmarks.metrics import main, quantile, timing_summary


def test_quantile_and_summary():
    assert quantile([4.0, 1.0, 3.0, 2.0], 0.5) == 2.5
    assert quantile([1.0, 2.0], 0.95) == pytest.approx(1.95)
    assert quantile([7.0], 0.3) == 7.0
    s = timing_summary([2.0, 1.0, 4.0], 100)
    assert s["elapsed_seconds"]["median"] == 2.0 and s["rows_per_second"]["median"] == 50.0
    with pytest.raises(ValueError):
        timing_summary([], 1)
    with pytest.raises(ValueError):
        quantile([1.0], 1.5)


def test_metric_benchmark_small_window(tmp_path, capsys):
    out = tmp_path / "m.json"
    assert main(["--batches", "2", "--rows-per-batch", "600", "--targets", "2", "--group-cardinality", "40",
                 "--ranks", "1,2", "--rounds", "1", "--device", "cpu", "--output", str(out)]) == 0
    got = json.loads(out.read_text())
    assert got["samples"] == 1200 and set(got["ranks"]) == {"1", "2"}
    assert got["max_abs_diff_merged_vs_local"] <= 1e-6
    assert 0.5 < got["metrics"]["auc_0"] < 1.0 and got["local"]["runs"] == 1
    assert json.loads(capsys.readouterr().out)["samples"] == 1200
