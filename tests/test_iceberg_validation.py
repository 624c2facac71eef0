"""Published-table checks on a local Iceberg table: physical schema and codec of every data file, row
counts against the manifests and duplicate data files in the scan (CPU)."""
import pytest

pa = pytest.importorskip("pyarrow")

from flare_b200.data.iceberg import IcebergSink, IcebergTable  # noqa: E402
from flare_b200.validation.iceberg import main, validate_physical_schema, validate_rows  # noqa: E402


def _table(tmp_path):
    data = pa.table({"a": list(range(100)), "b": [float(i) for i in range(100)], "_ds": ["2026-12-02"] * 100})
    t = IcebergTable.create(str(tmp_path / "t"), data.schema)
    IcebergSink(t).append([data.slice(0, 60), data.slice(60)])
    return t.refresh()


def test_schema_and_rows_of_a_published_table(tmp_path, capsys):
    t = _table(tmp_path)
    assert validate_physical_schema(t, ["a", "b", "_ds"]) == {"files": 2, "columns": 3, "codec": None}
    with pytest.raises(AssertionError, match=r"missing=\['c'\] unexpected=\['_ds'\]"):
        validate_physical_schema(t, ["a", "b", "c"])
    assert validate_physical_schema(t, ["a", "b", "_ds"], codec="zstd")["codec"] == "ZSTD"  # the sink's default
    snappy = IcebergTable.create(str(tmp_path / "s"), pa.schema([("a", pa.int64())]),
                                 properties={"write.parquet.compression-codec": "snappy"})
    IcebergSink(snappy).append([pa.table({"a": [1, 2, 3]})])
    with pytest.raises(AssertionError, match=r"only ZSTD compression.*SNAPPY"):
        validate_physical_schema(snappy.refresh(), ["a"], codec="zstd")
    assert validate_rows(t, 100) == {"rows": 100, "unique_data_files": 2}
    with pytest.raises(AssertionError, match="expected=99"):
        validate_rows(t, 99)
    assert main(["rows", t.location, "100"]) == 0
    assert main(["schema", t.location, "--columns", "a,b,_ds"]) == 0
    assert "iceberg_rows=100" in capsys.readouterr().out


def test_a_data_file_committed_twice_is_reported(tmp_path):
    t = _table(tmp_path)
    files = t.plan_files()
    t.append(files[:1])  # the same data file in a second snapshot
    with pytest.raises(AssertionError, match="twice"):
        validate_rows(t.refresh(), 160)
