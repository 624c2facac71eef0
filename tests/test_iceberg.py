"""Iceberg tables on the local filesystem (CPU): create / append / scan, idempotent commits, concurrent
committers, continuous-append cursors, orphan files, a lagging version hint, and the spec's manifest
field ids."""
import json

import pyarrow as pa
import pytest

from flare_b200.data import avro
from flare_b200.data.iceberg import (DataFile, IcebergSink, IcebergSourceFactory, IcebergTable)
from flare_b200.data.sources import stream_batches

SCHEMA = pa.schema([pa.field("label", pa.float32()), pa.field("d0", pa.float32()),
                    pa.field("s0", pa.list_(pa.int32())), pa.field("user", pa.string())])


def _batch(lo, n):
    return pa.table({"label": pa.array([float(i % 2) for i in range(lo, lo + n)], pa.float32()),
                     "d0": pa.array([i * 0.5 for i in range(lo, lo + n)], pa.float32()),
                     "s0": pa.array([[i, i + 1] for i in range(lo, lo + n)], pa.list_(pa.int32())),
                     "user": pa.array([f"u{i}" for i in range(lo, lo + n)])}, schema=SCHEMA)


def test_create_append_scan_and_read(tmp_path):
    t = IcebergTable.create(tmp_path / "tbl", SCHEMA)
    assert t.current_snapshot() is None and t.plan_files() == []
    sch = t.schema()
    assert [f["id"] for f in sch["fields"]] == [1, 2, 3, 5] and sch["fields"][2]["type"]["element-id"] == 4
    sink = IcebergSink(t)
    s1 = sink.append([_batch(0, 100), _batch(100, 50)], commit_id="w1")
    s2 = sink.append([_batch(150, 70)], commit_id="w2")
    assert s2["parent-snapshot-id"] == s1["snapshot-id"] and s2["sequence-number"] == 2
    files = t.plan_files()
    assert sum(f.record_count for f in files) == 220 and len(files) == 3
    assert sum(f.record_count for f in t.plan_files(s1["snapshot-id"])) == 150
    assert t.current_snapshot()["summary"]["total-records"] == "220"
    src = IcebergSourceFactory(IcebergTable.load(tmp_path / "tbl"), columns=["d0", "s0"])
    rows = []
    for ab in stream_batches(src, 64, policy="pad"):
        rows += ab.data.column("d0").to_pylist()[:ab.validity.valid_count]
    assert sorted(rows) == [i * 0.5 for i in range(220)]
    with pytest.raises(FileExistsError):
        IcebergTable.create(tmp_path / "tbl", SCHEMA)
    with pytest.raises(FileNotFoundError):
        IcebergTable.load(tmp_path / "none")


def test_commits_are_idempotent_and_recoverable(tmp_path):
    t = IcebergTable.create(tmp_path / "tbl", SCHEMA)
    sink = IcebergSink(t)
    a = sink.append([_batch(0, 10)], commit_id="input-7")
    b = sink.append([_batch(0, 10)], commit_id="input-7")  # a restarted writer repeats its commit
    assert a["snapshot-id"] == b["snapshot-id"] and len(t.refresh().snapshots()) == 1
    assert t.find_commit("input-7")["snapshot-id"] == a["snapshot-id"] and t.find_commit("x") is None
    # a writer that died after writing its files but before committing leaves orphans
    orphans = sink.write_files([_batch(10, 5)])
    assert t.orphan_files() == [t.io.resolve(orphans[0].path)[1]]


def test_concurrent_committers_both_land(tmp_path):
    IcebergTable.create(tmp_path / "tbl", SCHEMA)
    a, b = IcebergTable.load(tmp_path / "tbl"), IcebergTable.load(tmp_path / "tbl")
    fa = IcebergSink(a).write_files([_batch(0, 10)])
    fb = IcebergSink(b).write_files([_batch(10, 10)])
    a.append(fa, commit_id="a")
    b.append(fb, commit_id="b")  # b's table object is stale: its first try conflicts, then it re-reads
    t = IcebergTable.load(tmp_path / "tbl")
    assert t.version == 3 and len(t.snapshots()) == 2
    assert sum(f.record_count for f in t.plan_files()) == 20
    assert [s["summary"]["flare.commit-id"] for s in reversed(t.ancestry())] == ["a", "b"]


def test_continuous_append_cursor(tmp_path):
    t = IcebergTable.create(tmp_path / "tbl", SCHEMA)
    sink = IcebergSink(t)
    sink.append([_batch(0, 30)], commit_id="1")
    first = IcebergSourceFactory(t, mode="continuous", after_snapshot_id=None)
    assert sum(f.record_count for f in first.files) == 30
    sink.append([_batch(30, 20)], commit_id="2")
    sink.append([_batch(50, 5)], commit_id="3")
    nxt = IcebergSourceFactory(t.refresh(), mode="continuous", after_snapshot_id=first.cursor)
    assert [f.record_count for f in nxt.files] == [20, 5]
    again = IcebergSourceFactory(t, mode="continuous", after_snapshot_id=nxt.cursor)
    assert again.files == [] and again.plan() == []
    pinned = IcebergSourceFactory(t, mode="pinned", snapshot_id=first.cursor)
    assert sum(f.record_count for f in pinned.files) == 30


def test_lagging_version_hint_and_manifest_field_ids(tmp_path):
    t = IcebergTable.create(tmp_path / "tbl", SCHEMA)
    IcebergSink(t).append([_batch(0, 4)])
    (tmp_path / "tbl" / "metadata" / "version-hint.text").write_text("1")  # the hint update was lost
    t2 = IcebergTable.load(tmp_path / "tbl")
    assert t2.version == 2 and t2.current_snapshot() is not None
    snap = t2.current_snapshot()
    lst, meta = avro.read_container((tmp_path / "tbl" / "metadata" / snap["manifest-list"].split("/")[-1]).read_bytes())
    assert meta["format-version"] == b"2" and lst[0]["added_files_count"] == 1
    schema = json.loads(meta["avro.schema"])
    ids = {f["name"]: f["field-id"] for f in schema["fields"]}
    assert ids["manifest_path"] == 500 and ids["added_snapshot_id"] == 503 and ids["sequence_number"] == 515
    entries, _ = avro.read_container(open(lst[0]["manifest_path"], "rb").read())
    assert entries[0]["status"] == 1 and entries[0]["sequence_number"] is None  # inherited (v2)
    with pytest.raises(ValueError, match="at least one"):
        t2.append([])
    with pytest.raises(ValueError, match="ancestor"):
        t2.appended_files(12345)
    assert isinstance(DataFile("p", 1, 1), DataFile)


def test_pipeline_publishes_to_iceberg_and_recovers_a_missing_commit(tmp_path):
    from test_pipeline import _cfg, _write_logs

    from flare_b200.data.pipeline import DataPipeline
    from flare_b200.data.sources import StandardSourceFactory

    (tmp_path / "logs").mkdir()
    for i, n in enumerate([120, 80]):
        _write_logs(tmp_path / "logs" / f"f{i}.txt", n, 3 + i)
    cfg = _cfg(tmp_path, iceberg_table=str(tmp_path / "ice"))
    DataPipeline(cfg).run()
    t = IcebergTable.load(tmp_path / "ice")
    assert len(t.snapshots()) == 2 and sum(f.record_count for f in t.plan_files()) == 200
    # a crash between the pipeline's commit and the Iceberg commit: drop the last snapshot's metadata
    (tmp_path / "ice" / "metadata" / "v3.metadata.json").unlink()
    (tmp_path / "ice" / "metadata" / "version-hint.text").write_text("2")
    assert len(IcebergTable.load(tmp_path / "ice").snapshots()) == 1
    DataPipeline(cfg).run()  # nothing left to encode; reconciliation re-commits the missing input
    t = IcebergTable.load(tmp_path / "ice")
    assert len(t.snapshots()) == 2 and sum(f.record_count for f in t.plan_files()) == 200
    src = StandardSourceFactory.create("iceberg", {"table": str(tmp_path / "ice"), "columns": ["label"]})
    assert sum(it.rows for it in src.plan()) == 200
    with pytest.raises(ValueError, match="unknown"):
        StandardSourceFactory.create("iceberg", {"table": str(tmp_path / "ice"), "bogus": 1})
