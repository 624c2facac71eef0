"""Input-pipeline throughput harness (CPU): sink reports, summary validation, a small end-to-end run."""
import pytest

pa = pytest.importorskip("pyarrow")

from flare_b200.benchmarks.throughput import (  # noqa: E402
    ThroughputSink, run_throughput_benchmark, summarize_sink_reports, write_synthetic_parquet)


def _reports(steps=4, n=2, per=8):
    out = []
    for r in range(n):
        s = ThroughputSink(r, n, max_steps=steps)
        for _ in range(steps):
            s.consume(per)
        rep = s.report()
        rep["step_intervals"] = [0.5] * (steps - 1)
        rep["measured_duration_seconds"] = 0.5 * (steps - 1)
        out.append(rep)
    return out


def test_summary_numbers_and_validation():
    s = summarize_sink_reports(_reports(), input_workers=2, reader_workers=4, samples_per_input_step=8,
                               global_batch_size=16, steps=4, wall_seconds=2.0)
    assert s["valid_samples"] == 64 and s["end_to_end_aggregate_samples_per_second"] == 32.0
    assert s["arrival_window_samples"] == 48 and s["arrival_window_seconds"] == 1.5
    assert s["arrival_window_aggregate_samples_per_second"] == 32.0 and s["p95_step_seconds"] == 0.5
    assert s["reader_interleave_factor"] == 2
    with pytest.raises(ValueError):
        summarize_sink_reports(_reports(), input_workers=2, reader_workers=3, samples_per_input_step=8,
                               global_batch_size=16, steps=4, wall_seconds=2.0)
    bad = _reports()
    bad[1]["step_valid_samples"][0] = 7
    with pytest.raises(ValueError):
        summarize_sink_reports(bad, input_workers=2, reader_workers=4, samples_per_input_step=8,
                               global_batch_size=16, steps=4, wall_seconds=2.0)
    with pytest.raises(ValueError):
        summarize_sink_reports(_reports()[:1], input_workers=2, reader_workers=4, samples_per_input_step=8,
                               global_batch_size=16, steps=4, wall_seconds=2.0)


def test_small_run(tmp_path):
    paths = write_synthetic_parquet(str(tmp_path), files=2, rows_per_file=2048, num_sparse=4, num_dense=2,
                                    max_bag=4, row_group=512)
    s = run_throughput_benchmark(paths, input_workers=2, reader_workers=2, samples_per_input_step=512, steps=5,
                                 num_sparse=4, num_dense=2, rows_per_item=512)
    assert s["graph_steps"] == 5 and s["valid_samples"] == 5120
    assert s["end_to_end_aggregate_samples_per_second"] > 0
