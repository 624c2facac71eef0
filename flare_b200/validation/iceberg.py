"""Checks of a published Iceberg table's data files (the table format of ``data.iceberg``).

* ``validate_physical_schema``: every data file of the current snapshot has exactly the expected
  Parquet columns (the features plus whatever partition columns the publisher adds), reported as the
  missing and the unexpected names of the first file that differs; optionally every column chunk
  uses one compression codec (``codec="ZSTD"`` for tables whose writers must use zstd).
* ``validate_rows``: the scan plans no data file twice, the planned record counts add up to
  ``expected_rows``, and every file's own Parquet footer holds the record count its manifest entry
  claims.

    python -m flare_b200.validation.iceberg schema TABLE_LOCATION --columns a,b,c [--codec ZSTD]
    python -m flare_b200.validation.iceberg schema TABLE_LOCATION --manifest-dir PIPELINE_OUTPUT
    python -m flare_b200.validation.iceberg rows TABLE_LOCATION EXPECTED_ROWS

Reference behaviour: tools/validation/validate_iceberg.py (the physical schema of every planned data
file against the feature manifest with ZSTD-only column chunks; the row count and duplicate data files
of the scan), for tables reached through a REST catalog; these read the table's own metadata from
any location the object-store layer resolves.
"""
from __future__ import annotations

import argparse
from pathlib import Path

import pyarrow as pa
import pyarrow.parquet as pq

from ..data.iceberg import IcebergTable


def _footer(table: IcebergTable, path: str) -> pq.ParquetFile:
    return pq.ParquetFile(pa.BufferReader(table.io.read_bytes(path)))


def validate_physical_schema(table: IcebergTable, expected_columns, *, codec: str | None = None) -> dict:
    expected = set(expected_columns)
    files = table.plan_files()
    if not files:
        raise RuntimeError("the table's current snapshot has no data files")
    for f in files:
        pf = _footer(table, f.path)
        actual = set(pf.schema_arrow.names)
        missing, unexpected = sorted(expected - actual), sorted(actual - expected)
        if missing or unexpected:
            raise AssertionError(f"data file schema differs from the expected columns: path={f.path!r} "
                                 f"missing={missing!r} unexpected={unexpected!r}")
        if codec is not None:
            md = pf.metadata
            codecs = {md.row_group(g).column(c).compression for g in range(md.num_row_groups)
                      for c in range(md.row_group(g).num_columns)}
            if codecs != {codec.upper()}:
                raise AssertionError(f"data file must use only {codec.upper()} compression: path={f.path!r} "
                                     f"codecs={sorted(codecs)!r}")
    return {"files": len(files), "columns": len(expected), "codec": codec.upper() if codec else None}


def validate_rows(table: IcebergTable, expected_rows: int) -> dict:
    counts: dict[str, int] = {}
    for f in table.plan_files():
        if f.path in counts:
            raise AssertionError(f"the scan planned a data file twice: {f.path}")
        counts[f.path] = int(f.record_count)
        footer_rows = _footer(table, f.path).metadata.num_rows
        if footer_rows != f.record_count:
            raise AssertionError(f"{f.path}: the manifest says {f.record_count} rows, the file holds {footer_rows}")
    total = sum(counts.values())
    if total != expected_rows:
        raise AssertionError(f"row count differs: expected={expected_rows} actual={total}")
    return {"rows": total, "unique_data_files": len(counts)}


def _columns(arg: str) -> list[str]:
    p = Path(arg)
    if p.is_file():
        return [line.strip() for line in p.read_text().splitlines() if line.strip()]
    return [c for c in arg.split(",") if c]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="checks of a published Iceberg table's data files")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("schema")
    s.add_argument("location")
    g = s.add_mutually_exclusive_group(required=True)
    g.add_argument("--columns", help="comma-separated names, or a file with one name per line")
    g.add_argument("--manifest-dir", help="a directory with the feature pipeline's feature_manifest.json")
    s.add_argument("--extra-columns", default="", help="columns the publisher adds beyond the catalog")
    s.add_argument("--codec", default=None)
    r = sub.add_parser("rows")
    r.add_argument("location")
    r.add_argument("expected_rows", type=int)
    args = ap.parse_args(argv)
    table = IcebergTable.load(args.location)
    if args.cmd == "schema":
        if args.manifest_dir:
            from ..data.feature_catalog import FeatureCatalog

            cols = list(FeatureCatalog.from_manifest_dir(args.manifest_dir).columns)
        else:
            cols = _columns(args.columns)
        cols += [c for c in args.extra_columns.split(",") if c]
        out = validate_physical_schema(table, cols, codec=args.codec)
        print(f"physical_schema_files={out['files']} columns={out['columns']} compression={out['codec'] or 'any'}")
    else:
        out = validate_rows(table, args.expected_rows)
        print(f"iceberg_rows={out['rows']} unique_data_files={out['unique_data_files']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["validate_physical_schema", "validate_rows"]
