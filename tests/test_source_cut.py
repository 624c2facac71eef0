"""A checkpoint's reader cut: committed with the model state, restored at any world size so every input
row is read exactly once across the restart, and checked offline by the source-cut inspector (CPU)."""
import json
import os

import pytest
import torch

pa = pytest.importorskip("pyarrow")
pq = pytest.importorskip("pyarrow.parquet")

from flare_b200.checkpoint.source_cut import inspect_source_cut, load_reader_cut, main, save_reader_cut  # noqa: E402
from flare_b200.checkpoint.store import step_dir  # noqa: E402
from flare_b200.data.reader import BatchReader  # noqa: E402
from flare_b200.data.sources import ParquetSourceFactory  # noqa: E402

ALL = sorted(x for f in range(3) for x in range(f * 1000, f * 1000 + 100))


def _factory(tmp_path):
    paths = []
    for f in range(3):
        p = tmp_path / f"f{f}.parquet"
        pq.write_table(pa.table({"x": list(range(f * 1000, f * 1000 + 100))}), p, row_group_size=25)
        paths.append(str(p))
    return ParquetSourceFactory(paths)  # 12 items of 25 rows


def _ids(batches):
    return [v for b, val in batches for v in b.column("x").to_pylist()[:val.valid_count]]


def _take(reader, n):
    it = iter(reader)
    return _ids([next(it) for _ in range(n)])


def _engine_and_tables():
    import torch.nn as nn

    from flare_b200.recipes.cpu_small import SmallDense, small_tables
    from flare_b200.sparse.reference import CpuEmbeddingBagCollection
    from flare_b200.training.contracts import TrainingExecutionPlan
    from flare_b200.training.engine import TrainEngine
    from flare_b200.training.flat import DenseOptimizerConfig

    torch.manual_seed(0)
    engine = TrainEngine(SmallDense(), lambda out, y: nn.functional.binary_cross_entropy_with_logits(out, y),
                         TrainingExecutionPlan.replicated(), DenseOptimizerConfig(kind="adam", learning_rate=1e-3),
                         device=torch.device("cpu"))
    return engine, CpuEmbeddingBagCollection(small_tables(), 16, seed=0)


def test_cpu_checkpoint_commits_and_restores_the_reader_cut(tmp_path):
    from flare_b200.checkpoint.cpu import restore_cpu, save_cpu

    fac, root = _factory(tmp_path), tmp_path / "ckpt"
    engine, emb = _engine_and_tables()
    rd = BatchReader(fac, 30, policy="drop")
    before = _take(rd, 3)  # 90 rows: 3 whole items and 15 rows of the fourth
    save_cpu(root, 3, engine, emb, reader=rd)
    assert inspect_source_cut(root, 3, expected_readers=1)["partial_items"] == {"3": 15}
    engine2, emb2 = _engine_and_tables()
    rd2 = BatchReader(fac, 30, policy="pad")
    assert restore_cpu(root, engine2, emb2, reader=rd2) == 3
    after = _ids(list(rd2))
    assert sorted(before + after) == ALL and not set(before) & set(after)
    with pytest.raises(ValueError, match="no reader cut"):
        save_cpu(root, 4, engine, emb)
        restore_cpu(root, engine2, emb2, reader=BatchReader(fac, 30))


def test_two_rank_cut_resumes_on_three_ranks_and_inspects(tmp_path, capsys):
    fac, root = _factory(tmp_path), tmp_path / "ckpt"
    readers = [BatchReader(fac, 25, rank=r, world=2, policy="drop") for r in range(2)]
    got = [x for rd in readers for x in _take(rd, 3)]
    final = step_dir(root, 5)
    tmp = final.with_name(f"{final.name}.partial")
    for rd in readers:  # each rank writes its own file, then the commit renames the step into place
        save_reader_cut(tmp, 5, rd.capture_state())
    with pytest.raises(AssertionError, match="partial"):
        inspect_source_cut(root, 5)
    os.replace(tmp, final)
    out = inspect_source_cut(root, 5, expected_readers=2)
    assert out["readers"] == 2 and out["items_consumed"] == 6 and out["positions_consumed"] == 6
    assert main([str(root), "5", "--expected-readers", "2"]) == 0
    assert "checkpoint_source_cut_consistent=true" in capsys.readouterr().out
    rest = []
    for r in range(3):
        rd = BatchReader(fac, 25, rank=r, world=3, policy="drop")
        rd.restore_state(load_reader_cut(final))
        rest += _ids(list(rd))
    assert sorted(got + rest) == ALL and not set(got) & set(rest)


def test_inspector_rejects_inconsistent_cuts(tmp_path):
    fac, root = _factory(tmp_path), tmp_path / "ckpt"
    readers = [BatchReader(fac, 25, rank=r, world=2, policy="drop") for r in range(2)]
    for rd in readers:
        _take(rd, 2)
    d = step_dir(root, 7)
    for rd in readers:
        save_reader_cut(d, 7, rd.capture_state())
    with pytest.raises(AssertionError, match="expected 3"):
        inspect_source_cut(root, 7, expected_readers=3)
    f1 = d / "reader" / "rank1.json"
    rec = json.loads(f1.read_text())
    rec["state"]["done"] = rec["state"]["done"] + [json.loads((d / "reader" / "rank0.json").read_text())
                                                   ["state"]["done"][0]]
    f1.write_text(json.dumps(rec))
    with pytest.raises(AssertionError, match="consumed by ranks"):
        inspect_source_cut(root, 7)
    rec["step"] = 6
    f1.write_text(json.dumps(rec))
    with pytest.raises(AssertionError, match="cut of step 6"):
        inspect_source_cut(root, 7)
    f1.unlink()
    with pytest.raises(AssertionError, match="ranks"):
        inspect_source_cut(root, 7)
    with pytest.raises(AssertionError, match="not committed"):
        inspect_source_cut(root, 8)
