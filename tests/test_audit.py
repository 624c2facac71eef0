"""Checkpoint audit on a hand-written checkpoint in the store's format (CPU)."""
import json

import numpy as np

from flare_b200.checkpoint.audit import audit_step
from flare_b200.checkpoint.store import FORMAT_DENSE, FORMAT_SPARSE, step_dir


def _write(root, step, *, split_rows, nan=False, drop_piece=False):
    d = step_dir(root, step)
    (d / "model").mkdir(parents=True)
    rng = np.random.default_rng(0)
    w = rng.normal(size=(4, 3)).astype(np.float32)
    for f in ("master", "m", "v"):
        np.save(d / "model" / f"fc.{f}.npy", np.abs(w) if f == "v" else w)
    (d / "model" / "manifest.json").write_text(json.dumps({"format": FORMAT_DENSE, "step": step, "optimizer_step": 5,
                                                           "optimizer": "adam",
                                                           "entries": {"fc": {"shape": [4, 3], "dtype": "float32"}}}))
    sp = d / "sparse" / "tables"
    sp.mkdir(parents=True)
    table = rng.normal(size=(10, 8)).astype(np.float32)
    state = np.abs(rng.normal(size=10)).astype(np.float32)
    if nan:
        table[3, 2] = np.nan
    pieces = []
    if split_rows:
        for r in range(2):
            if drop_piece and r == 1:
                continue
            np.save(sp / f"t.c0.r{r}of2.weight.npy", table[r::2])
            np.save(sp / f"t.c0.r{r}of2.state_row.npy", state[r::2])
            pieces.append({"table": "t", "col_begin": 0, "ncols": 8, "rank": r, "row_index": r, "row_shards": 2})
    else:
        for cb in (0, 4):
            np.save(sp / f"t.c{cb}.weight.npy", table[:, cb:cb + 4])
            np.save(sp / f"t.c{cb}.state_row.npy", state)
            pieces.append({"table": "t", "col_begin": cb, "ncols": 4, "rank": cb // 4, "row_index": 0, "row_shards": 1})
    (sp / "manifest.json").write_text(json.dumps({
        "format": FORMAT_SPARSE, "step": step, "mode": "full", "base_step": None, "optimizer": "rowwise_adagrad",
        "optimizer_step": 5, "tables": [{"name": "t", "rows": 10, "dim": 8, "value_dtype": "float32",
                                         "pooling": "sum"}], "pieces": pieces, "world_size": 2}))


def test_audit_digest_independent_of_sharding(tmp_path):
    _write(tmp_path / "a", 1, split_rows=True)
    _write(tmp_path / "b", 1, split_rows=False)
    a, b = audit_step(tmp_path / "a"), audit_step(tmp_path / "b")
    assert a["ok"] and b["ok"]
    assert a["sparse"]["digest"] == b["sparse"]["digest"] and a["dense"]["digest"] == b["dense"]["digest"]


def test_audit_reports_problems(tmp_path):
    _write(tmp_path / "n", 1, split_rows=True, nan=True)
    assert not audit_step(tmp_path / "n")["ok"]
    _write(tmp_path / "d", 1, split_rows=True, drop_piece=True)
    rep = audit_step(tmp_path / "d")
    assert not rep["ok"] and any("cover" in p for p in rep["sparse"]["problems"])


def test_checkpoint_reads_retry_transient_errors(tmp_path, monkeypatch):
    import numpy as np
    import pytest

    from flare_b200.checkpoint import store

    np.save(tmp_path / "a.npy", np.arange(3))
    real, calls = np.load, []

    def flaky(path, *a, **k):
        calls.append(path)
        if len(calls) < 3:
            raise OSError("transient")
        return real(path, *a, **k)

    monkeypatch.setattr(store.np, "load", flaky)
    assert store._read_array(tmp_path / "a.npy").tolist() == [0, 1, 2] and len(calls) == 3
    calls.clear()
    monkeypatch.setattr(store.np, "load", lambda *a, **k: (_ for _ in ()).throw(OSError("down")))
    with pytest.raises(OSError):
        store._read_array(tmp_path / "a.npy")
