"""Exactly-once Iceberg publication across real process crashes (os._exit before and after the metadata
commit): the re-run publishes each window once, and a crash before the commit leaves only orphan data
files (CPU, subprocess workers)."""
import subprocess
import sys
from pathlib import Path

from flare_b200.data.iceberg import IcebergTable
from flare_b200.validation.iceberg import validate_rows

ROOT = Path(__file__).resolve().parents[1]


def _run(table, window, mode):
    return subprocess.run([sys.executable, "-m", "flare_b200.testing.iceberg_crash", str(table), str(window), mode],
                          cwd=ROOT, capture_output=True, text=True, timeout=300)


def _ids(t):
    import pyarrow.parquet as pq

    return sorted(i for f in t.plan_files() for i in pq.read_table(f.path, columns=["id"]).column("id").to_pylist())


def test_crash_before_the_commit_then_rerun_publishes_once(tmp_path):
    table = tmp_path / "t"
    assert _run(table, 0, "clean").returncode == 0
    r = _run(table, 1, "before")
    assert r.returncode == 85, r.stderr
    t = IcebergTable.load(table)
    assert len(t.snapshots()) == 1 and len(t.orphan_files()) == 1  # window 1's data file, never committed
    assert _run(table, 1, "clean").returncode == 0
    t = IcebergTable.load(table)
    assert [s["summary"].get("flare.commit-id") for s in t.snapshots()] == ["window-0", "window-1"]
    assert _ids(t) == list(range(200)) and validate_rows(t, 200)["unique_data_files"] == 2


def test_crash_after_the_commit_then_rerun_does_not_publish_again(tmp_path):
    table = tmp_path / "t"
    r = _run(table, 3, "after")
    assert r.returncode == 86, r.stderr
    assert len(IcebergTable.load(table).snapshots()) == 1  # the commit happened before the exit
    rerun = _run(table, 3, "clean")
    assert rerun.returncode == 0, rerun.stderr
    t = IcebergTable.load(table)
    assert len(t.snapshots()) == 1 and _ids(t) == list(range(300, 400)) and not t.orphan_files()
