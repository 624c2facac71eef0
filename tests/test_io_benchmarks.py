"""I/O-path benchmarks on a local directory: an Iceberg table read through the connector's file IO and
directly returns the same rows; append commits publish exactly the rows written."""
import json

from flare_b200.benchmarks.io_paths import bench_reads, bench_writes, main, make_table, synthetic_rows


def test_synthetic_rows_are_deterministic():
    a, b = synthetic_rows(10, 3), synthetic_rows(10, 3)
    assert a.equals(b) and a.num_columns == 3 and a.column("row_id").to_pylist() == list(range(10))


def test_read_benchmark_on_a_local_table(tmp_path):
    loc = str(tmp_path / "t")
    t = make_table(loc, files=3, rows_per_file=200, columns=4)
    assert sum(f.record_count for f in t.plan_files()) == 600
    out = bench_reads(loc, projection_count=2, concurrency=2, repetitions=2)
    assert out["files"] == 3 and out["rows"] == 600 and out["projection"] == ["row_id", "f1"]
    assert out["table_io"]["runs"] == 2 and out["direct"]["rows_per_second"]["median"] > 0


def test_write_benchmark_commits_every_row(tmp_path, capsys):
    out = bench_writes(str(tmp_path / "w"), rows=1000, blocks=3, concurrency=2, repetitions=1, columns=3)
    assert out["blocks"] == 3 and out["iceberg_append"]["rows"] == 1000 and out["direct_parquet"]["runs"] == 1
    assert main(["make-table", str(tmp_path / "m"), "--files", "2", "--rows-per-file", "50", "--columns", "2"]) == 0
    assert json.loads(capsys.readouterr().out)["rows"] == 100
