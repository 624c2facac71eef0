"""Offline audit of a feature-pipeline output: a clean publication passes with the right totals; a
missing part file, a row-count mismatch, a column the catalog does not list and a crashed run's
temporary window are each reported (CPU)."""
import json

import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from flare_b200.data.pipeline import DataPipeline
from flare_b200.data.publication_audit import audit_publication, main


def _publish(tmp_path):
    from test_pipeline import _cfg, _write_logs

    (tmp_path / "logs").mkdir()
    for i, n in enumerate([150, 90]):
        _write_logs(tmp_path / "logs" / f"f{i}.txt", n, 7 + i)
    DataPipeline(_cfg(tmp_path)).run()
    return tmp_path / "out"


def test_clean_publication_passes(tmp_path, capsys):
    out = _publish(tmp_path)
    got = audit_publication(out)
    assert got["rows"] == 240 and got["inputs_done"] == 2 and got["temporary"] == []
    assert got["catalog_columns"] == ["d0", "label", "s0", "s1", "s2"]
    assert main([str(out)]) == 0 and json.loads(capsys.readouterr().out)["rows"] == 240


def test_inconsistencies_are_reported(tmp_path):
    out = _publish(tmp_path)
    man = json.loads((out / "_publication.json").read_text())
    first = out / man["windows"][0]["dir"] / "part-00000.parquet"
    table = pq.read_table(first)
    pq.write_table(table.slice(1), first)  # one row lost
    with pytest.raises(AssertionError, match="rows, its manifest entry says"):
        audit_publication(out)
    pq.write_table(table.append_column("extra", pa.array([0] * table.num_rows)), first)
    with pytest.raises(AssertionError, match=r"unexpected \['extra'\]"):
        audit_publication(out)
    pq.write_table(table, first)
    (out / ".window-crashed").mkdir()
    with pytest.raises(AssertionError, match="temporary windows"):
        audit_publication(out)
    assert audit_publication(out, allow_temporary=True)["temporary"] == [".window-crashed"]
    first.unlink()
    with pytest.raises(AssertionError, match="holds"):
        audit_publication(out, allow_temporary=True)
