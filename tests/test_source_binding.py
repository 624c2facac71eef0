"""Dataset source binding (CPU): reader topology from an execution cycle, tail layout per completion
policy, plan identity, round-robin / contiguous assignment, and per-rank readers over Parquet."""
import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from flare_b200.data.source_binding import (AssignmentPolicy, ScheduledDatasetSource, TailLayoutMode,
                                            tail_layout_mode)
from flare_b200.data.sources import ParquetSourceFactory


@pytest.fixture
def factory(tmp_path):
    paths = []
    for f in range(3):
        t = pa.table({"x": list(range(f * 100, f * 100 + 100)), "y": [float(i) for i in range(100)]})
        p = tmp_path / f"part{f}.parquet"
        pq.write_table(t, p, row_group_size=25)
        paths.append(str(p))
    return ParquetSourceFactory(paths, rows_per_item=25)


def test_tail_layout_per_completion_policy():
    assert tail_layout_mode("drop") is TailLayoutMode.DISCARD_REMAINDER
    assert tail_layout_mode("carry") is TailLayoutMode.RETAIN_PENDING
    assert tail_layout_mode("require") is TailLayoutMode.REJECT_REMAINDER
    assert tail_layout_mode("pad") is TailLayoutMode.SYNTHESIZE_PADDING
    assert tail_layout_mode("drop_remainder") is TailLayoutMode.DISCARD_REMAINDER


def test_reader_topology(factory):
    src = ScheduledDatasetSource(factory, 64, "pad", job_id="j")
    topo = src.build_reader_topology(4, node_ids=["a", "a", "b", "b"])
    assert topo.execution_cycle == ((0, 1, 2, 3),) and topo.rows_per_reader() == 16
    assert topo.groups[2].worker_id == "j/reader/2" and topo.groups[2].node_id == "b"
    # alternating halves: two readers active per step, each with half of the global batch
    topo2 = src.build_reader_topology(4, cycle=[(0, 1), (2, 3)])
    assert topo2.rows_per_reader() == 32 and topo2.active_readers(3) == (2, 3)
    with pytest.raises(ValueError, match="uniform"):
        src.build_reader_topology(4, cycle=[(0, 1), (2,)])
    with pytest.raises(ValueError, match="divide"):
        ScheduledDatasetSource(factory, 66).build_reader_topology(4)
    with pytest.raises(ValueError, match="outside"):
        src.build_reader_topology(2, cycle=[(0, 5)])
    with pytest.raises(ValueError, match="positive"):
        ScheduledDatasetSource(factory, 0)
    with pytest.raises(TypeError):
        ScheduledDatasetSource(object(), 8)


def test_scan_binding_identity_and_assignments(factory, tmp_path):
    rr = ScheduledDatasetSource(factory, 33).build_scan_binding(3)
    assert len(rr.items) == 12 and rr.initial_cursor == 0
    assert rr.assignments[1] == (1, 4, 7, 10)
    assert sorted(i for a in rr.assignments for i in a) == list(range(12))
    rr.check_identity(ScheduledDatasetSource(factory, 33).build_scan_binding(3).identity)
    other = ParquetSourceFactory(factory.paths[:2], rows_per_item=25)
    with pytest.raises(ValueError, match="identity"):
        rr.check_identity(ScheduledDatasetSource(other, 33).build_scan_binding(3).identity)
    ct = ScheduledDatasetSource(factory, 33, assignment_policy="contiguous").build_scan_binding(3)
    assert ct.assignment_policy is AssignmentPolicy.CONTIGUOUS
    assert [len(a) for a in ct.assignments] == [4, 4, 4] and ct.assignments[0] == (0, 1, 2, 3)
    with pytest.raises(ValueError, match="assignment"):
        ScheduledDatasetSource(factory, 32, assignment_policy="random")


def test_readers_cover_the_dataset(factory):
    src = ScheduledDatasetSource(factory, 40, "pad")
    seen, padded = [], 0
    for r in range(2):
        reader = src.create_reader(r, 2)
        for batch, validity in reader:
            assert batch.num_rows == 20
            n = validity.valid_count if hasattr(validity, "valid_count") else int(validity)
            seen += batch.column("x").to_pylist()[:n]
            padded += 20 - n
    assert sorted(seen) == list(range(300))
    assert padded == 20  # 150 rows per rank: 7 full batches and one of 10 valid rows each
