"""Per-rank batch reader: assignment, cut-position resume across world sizes, repeat mode, audit (CPU)."""
import json

import pytest

pa = pytest.importorskip("pyarrow")
pq = pytest.importorskip("pyarrow.parquet")

from flare_b200.data.reader import BatchReader, global_valid_count  # noqa: E402
from flare_b200.data.sources import ParquetSourceFactory  # noqa: E402


def _files(tmp_path, n_files=3, rows=100):
    paths = []
    for f in range(n_files):
        p = tmp_path / f"f{f}.parquet"
        pq.write_table(pa.table({"x": list(range(f * 1000, f * 1000 + rows))}), p, row_group_size=25)
        paths.append(str(p))
    return paths


def _ids(batches):
    return [v for b, val in batches for v in b.column("x").to_pylist()[:val.valid_count]]


def test_ranks_partition_the_items_and_audit(tmp_path):
    fac = ParquetSourceFactory(_files(tmp_path))  # 12 items of 25 rows
    seen = []
    for r in range(2):
        rd = BatchReader(fac, 16, rank=r, world=2, audit_path=tmp_path / f"audit{r}.json")
        seen += _ids(list(rd))
        rd.close()
    assert sorted(seen) == sorted(x for f in range(3) for x in range(f * 1000, f * 1000 + 100))
    a = json.loads((tmp_path / "audit0.json").read_text())
    assert a["items"] == 6 and a["rows"] == 150 and a["padded_rows"] == 10


def test_resume_with_a_different_world(tmp_path):
    fac = ParquetSourceFactory(_files(tmp_path))
    readers = [BatchReader(fac, 25, rank=r, world=2, policy="drop") for r in range(2)]
    got = []
    for rd in readers:  # each rank consumes 3 batches (3 whole items) and stops
        it = iter(rd)
        got += _ids([next(it) for _ in range(3)])
    states = [rd.capture_state() for rd in readers]
    rest = []
    for r in range(3):  # resume on 3 ranks
        rd = BatchReader(fac, 25, rank=r, world=3, policy="drop")
        rd.restore_state(states)
        rest += _ids(list(rd))
    assert sorted(got + rest) == sorted(x for f in range(3) for x in range(f * 1000, f * 1000 + 100))
    assert not set(got) & set(rest)


def test_repeat_first_batch_and_global_count(tmp_path):
    rd = BatchReader(ParquetSourceFactory(_files(tmp_path, 1)), 10, repeat_first_batch=True)
    it = iter(rd)
    a, b = next(it), next(it)
    assert a[0].column("x").to_pylist() == b[0].column("x").to_pylist()
    assert global_valid_count(10, expected=10) == 10
    with pytest.raises(RuntimeError):
        global_valid_count(9, expected=10)


def test_cut_position_inside_an_item(tmp_path):
    fac = ParquetSourceFactory(_files(tmp_path, 2))  # 8 items of 25 rows
    rd = BatchReader(fac, 10, rank=0, world=1, policy="pad")
    it = iter(rd)
    got = _ids([next(it) for _ in range(4)])  # 40 rows: items 0 (25) done, item 1 cut at 15
    st = rd.capture_state()
    assert st["done"] == [0] and st["current"] == [1, 15]
    rd2 = BatchReader(fac, 10, rank=0, world=1, policy="pad")
    rd2.restore_state([st])
    rest = _ids(list(rd2))
    assert sorted(got + rest) == sorted(x for f in range(2) for x in range(f * 1000, f * 1000 + 100))


def test_reconcile_reader_audits(tmp_path):
    from flare_b200.data.reader import main, reconcile_reader_audits

    fac = ParquetSourceFactory(_files(tmp_path))
    audits = []
    for r in range(3):
        rd = BatchReader(fac, 16, rank=r, world=3, audit_path=tmp_path / f"a{r}.json")
        list(rd)
        audits.append(rd.close())
    items = [it.item_id for it in fac.plan()]
    rep = reconcile_reader_audits(audits, items, planned_rows=300)
    assert rep["ok"] and rep["items_consumed"] == 12 and rep["rows"] == 300
    bad = [dict(audits[0]), audits[1]]  # rank 2's audit lost, rank 0 also claims one of rank 1's items
    bad[0]["done"] = bad[0]["done"] + [audits[1]["done"][0]]
    rep = reconcile_reader_audits(bad, items, planned_rows=300)
    assert not rep["ok"] and rep["duplicated"] == [audits[1]["done"][0]]
    assert rep["missing"] == sorted(audits[2]["done"]) and not rep["ranks_complete"]
    assert main([str(tmp_path / f"a{r}.json") for r in range(3)] + ["--items", "12", "--rows", "300"]) == 0


def test_parquet_range_batch_loader_shards_epochs_and_tail(tmp_path):
    from flare_b200.data.sources import ParquetRangeBatchLoader

    d = tmp_path / "ds"
    d.mkdir()
    for f in range(2):
        pq.write_table(pa.table({"x": list(range(f * 100, f * 100 + 100)), "y": [0] * 100}), d / f"p{f}.parquet",
                       row_group_size=25)
    seen, valid = [], 0
    for shard in range(2):
        ld = ParquetRangeBatchLoader(dataset_path=str(d), projection=["x"], batch_size=32,
                                     batch_transformer=lambda t: t, shard_index=shard, shard_count=2, num_epochs=2)
        for t in ld:
            assert t.column_names == ["x"] and t.num_rows == 32
            n = ld.last_validity.valid_count
            seen += t.column("x").to_pylist()[:n]
            valid += n
    assert valid == 400 and sorted(seen) == sorted(list(range(200)) * 2)
    with pytest.raises(ValueError, match="shard_index"):
        ParquetRangeBatchLoader(dataset_path=str(d), projection=["x"], batch_size=8, batch_transformer=len,
                                shard_index=2, shard_count=2)


def test_streaming_batch_reader_resumes_from_replay_ranges():
    from flare_b200.data.sources import StreamingBatchReader

    frags = {f"r{i}": pa.table({"x": list(range(i * 10, i * 10 + 10))}) for i in range(5)}

    def run(reader, names, first_skip=0):
        out = []
        for j, n in enumerate(names):
            t = frags[n].slice(first_skip) if j == 0 and first_skip else frags[n]
            out += [b.column("x").to_pylist() for b in reader.append_fragment(t, n)]
        return out

    whole = run(StreamingBatchReader(batch_size=16), list(frags))
    a = StreamingBatchReader(batch_size=16, validity_field="valid")
    head = run(a, ["r0", "r1"])
    state = a.checkpoint_state()
    assert state == {"pending_rows": 4, "replay": [["r1", 6]]}
    b = StreamingBatchReader(batch_size=16)
    b.restore_state(state)
    (rng, skip), = b.replay_ranges
    tail = run(b, [rng, "r2", "r3", "r4"], first_skip=skip)
    assert head + tail == whole and len(whole) == 3
    last = StreamingBatchReader(batch_size=16, completion_policy="pad", validity_field="valid")
    run(last, ["r0"])
    (t,) = last.finalize()
    assert t.num_rows == 16 and t.schema.metadata[b"valid"] == b"10"
