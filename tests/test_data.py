"""Schema, ragged batches, completion policies, range reads, synthetic generators and the prefetch loader (CPU)."""
import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from flare_b200.data.loader import PrefetchLoader
from flare_b200.data.schema import RaggedFeatureBatch, TrainingFeatureLayout, keyed_jagged_from_lists, \
    table_to_training_dict, virtual_pad
from flare_b200.data.sources import (BatchAssembler, CompletionPolicy, RecordRange, StandardSourceFactory,
                                     coalesce_source_ranges, stream_batches)
from flare_b200.data.synthetic import SparseBatch


def _table(n, seed=0):
    rng = np.random.default_rng(seed)
    ids = [list(rng.integers(0, 100, rng.integers(0, 4))) for _ in range(n)]
    ids[1] = None
    return pa.table({
        "uid": pa.array(rng.integers(0, 10, n)),
        "cat": pa.array([None if i % 5 == 0 else int(i % 7) for i in range(n)], pa.int64()),
        "x": pa.array(rng.random(n).astype(np.float32)),
        "hist": pa.array(ids, pa.list_(pa.int64())),
        "label": pa.array((rng.random(n) < 0.3).astype(np.float32)),
    })


def test_ragged_validation():
    RaggedFeatureBatch(np.arange(5), (np.array([0, 2, 5], np.int32),))
    with pytest.raises(ValueError):
        RaggedFeatureBatch(np.arange(5), (np.array([0, 3, 2], np.int32),))
    with pytest.raises(TypeError):
        RaggedFeatureBatch(np.arange(5), (np.array([0, 5]),))


def test_table_to_training_dict_and_pad():
    t = _table(10)
    layout = TrainingFeatureLayout({"cat": "cat", "x": "x", "hist": "hist"}, categorical=("cat",), dense=("x",))
    td = table_to_training_dict(t, layout, sparse_groups={"g": ["hist"]}, label_column="label",
                                metadata_columns=("uid",))
    assert td.side_info[0, 0] == 0 and td.side_info[1, 0] == 2  # null -> 0, value v -> v+1
    off, vals = td.sparse["g"]
    assert len(off) == 11 and off[2] - off[1] == 0 and len(vals) == off[-1]
    padded, valid = virtual_pad(td, 16)
    assert valid == 10 and padded.labels.shape == (16, 1) and len(padded.sparse["g"][0]) == 17
    o, v = keyed_jagged_from_lists([[[1, 2], [3]], [[4], []]])
    assert o.tolist() == [0, 2, 3, 4, 4] and v.tolist() == [1, 2, 3, 4]


def test_ranges_and_completion_policies(tmp_path):
    assert coalesce_source_ranges([RecordRange("a", 5, 9), RecordRange("a", 0, 5), RecordRange("b", 0, 1)]) == [
        RecordRange("a", 0, 9), RecordRange("b", 0, 1)]
    for i in range(2):
        pq.write_table(_table(37, seed=i), tmp_path / f"p{i}.parquet", row_group_size=10)
    fac = StandardSourceFactory.create("parquet", {"paths": str(tmp_path), "rows_per_item": 7})
    items = fac.plan()
    assert sum(it.rows for it in items) == 74
    batches = list(stream_batches(fac, 16, policy="pad"))
    assert len(batches) == 5 and batches[-1].validity.valid_count == 74 - 64
    assert len(list(stream_batches(fac, 16, policy="drop"))) == 4
    with pytest.raises(ValueError):
        list(stream_batches(fac, 16, policy="require"))
    asm = BatchAssembler(4, CompletionPolicy.from_value("drop_remainder"))
    out = asm.push({"a": np.arange(10)})
    assert [b.data["a"].tolist() for b in out] == [[0, 1, 2, 3], [4, 5, 6, 7]] and asm.finish() == []
    with pytest.raises(ValueError):
        StandardSourceFactory.create("iceberg-nope", {"paths": "x"})


def test_prefetch_loader_cpu():
    import torch

    def gen():
        for i in range(5):
            yield SparseBatch(torch.full((2, 3), float(i)), torch.zeros(2, 1), torch.tensor([0, 1, 2], dtype=torch.int32),
                              torch.tensor([i, i], dtype=torch.int32))

    got = [int(b.values[0]) for b in PrefetchLoader(gen(), depth=2)]
    assert got == [0, 1, 2, 3, 4]


def test_prefetch_loader_close_stops_the_worker_early():
    import itertools
    import time

    import torch

    made = []

    def endless():
        for i in itertools.count():
            made.append(i)
            yield SparseBatch(torch.zeros(1, 1), torch.zeros(1, 1), torch.tensor([0, 1], dtype=torch.int32),
                              torch.tensor([i], dtype=torch.int32))

    with PrefetchLoader(endless(), depth=2, pin_memory=False) as loader:
        it = iter(loader)
        assert [int(next(it).values[0]) for _ in range(3)] == [0, 1, 2]
    t0 = time.monotonic()
    loader._thread.join(timeout=2.0)
    assert not loader._thread.is_alive() and time.monotonic() - t0 < 2.0
    n = len(made)
    time.sleep(0.2)
    assert len(made) == n  # the source is no longer pulled


def test_prefetch_loader_reports_a_source_error():
    import pytest
    import torch

    def broken():
        yield SparseBatch(torch.zeros(1, 1), torch.zeros(1, 1), torch.tensor([0, 1], dtype=torch.int32),
                          torch.tensor([7], dtype=torch.int32))
        raise RuntimeError("source failed")

    it = iter(PrefetchLoader(broken(), depth=2, pin_memory=False))
    assert int(next(it).values[0]) == 7
    with pytest.raises(RuntimeError, match="source failed"):
        next(it)
