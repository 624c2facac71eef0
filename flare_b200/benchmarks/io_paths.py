"""Data-path I/O benchmarks: Iceberg reads and append commits against direct Parquet I/O.

    # make a table to read (any URI the object-store layer resolves; a local path here)
    python -m flare_b200.benchmarks.io_paths make-table /data/t --files 16 --rows-per-file 100000 --columns 8
    # read every data file of the current snapshot: through the table's file IO vs directly
    python -m flare_b200.benchmarks.io_paths reads /data/t --projection-count 4 --concurrency 8 --repetitions 3
    # publish rows: Iceberg append commits vs plain Parquet writes of the same blocks
    python -m flare_b200.benchmarks.io_paths writes /data/w --rows 1000000 --blocks 8 --concurrency 8 --repetitions 3

``reads`` plans the snapshot's data files (``data.iceberg.IcebergTable.plan_files``) and reads the
first ``projection-count`` columns of every file with ``concurrency`` threads, two ways:
``table_io`` (whole objects through ``io.objectstore.ObjectStoreIO``, the path the connector uses,
with its retries) and ``direct`` (pyarrow's own filesystem streams).  Both must return the same Arrow
data in every repetition.  ``writes`` publishes ``rows`` synthetic rows in ``blocks`` blocks per
repetition: ``iceberg_append`` writes the blocks as data files and commits them as one append
snapshot of a fresh table (manifest, manifest list, metadata commit), ``direct_parquet`` writes the
same blocks as Parquet files only; the committed snapshot's record count is checked.  Each prints
one JSON summary (median / p50 / p95 seconds and rows per second, ``benchmarks.metrics.timing_summary``)
and can write it to ``--output``.

Reference counterpart: tools/validation/benchmark_source_reads.py (Iceberg table IO vs direct S3
reads) and tools/validation/benchmark_publish_writes.py (Iceberg append commits vs direct S3 Parquet
writes), which need a REST catalog and S3; these run against any location the object-store layer
resolves, a local directory included.
"""
from __future__ import annotations

import argparse
import json
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq

from ..data.iceberg import DataFile, IcebergSink, IcebergTable
from ..io.objectstore import ObjectStoreIO
from .metrics import timing_summary


def synthetic_rows(rows: int, columns: int, offset: int = 0) -> pa.Table:
    """``row_id`` int64 plus ``columns - 1`` float32 feature columns, deterministic in the row id."""
    if rows <= 0 or columns <= 0:
        raise ValueError("rows and columns must be positive")
    ids = np.arange(offset, offset + rows, dtype=np.int64)
    cols = {"row_id": pa.array(ids)}
    for c in range(1, columns):
        cols[f"f{c}"] = pa.array(((ids * 2654435761 + c) % 1000).astype(np.float32) / np.float32(1000.0))
    return pa.table(cols)


def make_table(location: str, *, files: int, rows_per_file: int, columns: int, io=None) -> IcebergTable:
    """A fresh Iceberg table at ``location`` with ``files`` data files in one append snapshot."""
    if files <= 0:
        raise ValueError("files must be positive")
    first = synthetic_rows(rows_per_file, columns)
    table = IcebergTable.create(location, first.schema, io=io)
    blocks = [first] + [synthetic_rows(rows_per_file, columns, k * rows_per_file) for k in range(1, files)]
    IcebergSink(table).append(blocks)
    return table


def _parallel(fn, items, concurrency: int) -> list:
    if concurrency < 1:
        raise ValueError("concurrency must be positive")
    with ThreadPoolExecutor(max_workers=concurrency) as ex:
        return list(ex.map(fn, items))


def bench_reads(location: str, *, projection_count: int, concurrency: int, repetitions: int, io=None) -> dict:
    if repetitions < 1:
        raise ValueError("repetitions must be positive")
    table = IcebergTable.load(location, io=io)
    files = table.plan_files()
    if not files:
        raise RuntimeError("the table's current snapshot has no data files")
    names = table.arrow_schema().names
    if not 1 <= projection_count <= len(names):
        raise ValueError(f"projection count must be between 1 and {len(names)}")
    cols = names[:projection_count]
    rows = sum(f.record_count for f in files)
    store = table.io

    def via_table_io(f: DataFile) -> pa.Table:
        return pq.read_table(pa.BufferReader(store.read_bytes(f.path)), columns=cols)

    def direct(f: DataFile) -> pa.Table:
        fs, inner, _ = store.resolve(f.path)
        with fs.open_input_file(inner) as stream:
            return pq.read_table(stream, columns=cols)

    out = {"table": table.location, "files": len(files), "rows": rows, "projection": cols,
           "concurrency": concurrency}
    reference = None
    for label, read_one in (("table_io", via_table_io), ("direct", direct)):
        secs = []
        for _ in range(repetitions):
            t0 = time.perf_counter()
            parts = _parallel(read_one, files, concurrency)
            secs.append(time.perf_counter() - t0)
            got = pa.concat_tables(parts).combine_chunks()
            if reference is None:
                reference = got
            elif not got.equals(reference):
                raise AssertionError(f"{label} returned different Arrow data")
        out[label] = timing_summary(secs, rows)
    return out


def bench_writes(root: str, *, rows: int, blocks: int, concurrency: int, repetitions: int, columns: int = 4,
                 io=None) -> dict:
    if repetitions < 1 or blocks < 1:
        raise ValueError("repetitions and blocks must be positive")
    store = io or ObjectStoreIO()
    data = synthetic_rows(rows, columns)
    per = (rows + blocks - 1) // blocks
    parts = [data.slice(k * per, per) for k in range(blocks) if k * per < rows]
    base = str(root).rstrip("/")
    fs, inner_root, scheme = store.resolve(base)
    if scheme == "file":
        Path(inner_root).mkdir(parents=True, exist_ok=True)
    out = {"root": base, "rows": rows, "blocks": len(parts), "concurrency": concurrency}

    secs = []
    for r in range(repetitions):
        table = IcebergTable.create(f"{base}/iceberg-{r}-{time.time_ns()}", data.schema, io=store)
        sink = IcebergSink(table)
        t0 = time.perf_counter()
        files = [f for group in _parallel(lambda p: sink.write_files([p]), parts, concurrency) for f in group]
        snap = table.append(files)
        secs.append(time.perf_counter() - t0)
        if int(snap["summary"]["total-records"]) != rows:
            raise AssertionError(f"committed {snap['summary']['total-records']} rows, wrote {rows}")
    out["iceberg_append"] = timing_summary(secs, rows)

    secs = []
    for r in range(repetitions):
        d = f"{inner_root}/parquet-{r}-{time.time_ns()}"
        if scheme == "file":
            Path(d).mkdir(parents=True, exist_ok=True)

        def write_one(item, d=d):
            k, part = item
            with fs.open_output_stream(f"{d}/part-{k:05d}.parquet") as stream:
                pq.write_table(part, stream)

        t0 = time.perf_counter()
        _parallel(write_one, list(enumerate(parts)), concurrency)
        secs.append(time.perf_counter() - t0)
    out["direct_parquet"] = timing_summary(secs, rows)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Iceberg reads / append commits against direct Parquet I/O")
    sub = ap.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("make-table")
    m.add_argument("location")
    m.add_argument("--files", type=int, default=16)
    m.add_argument("--rows-per-file", type=int, default=100_000)
    m.add_argument("--columns", type=int, default=8)
    r = sub.add_parser("reads")
    r.add_argument("location")
    r.add_argument("--projection-count", type=int, default=4)
    r.add_argument("--concurrency", type=int, default=8)
    r.add_argument("--repetitions", type=int, default=3)
    r.add_argument("--output", type=Path)
    w = sub.add_parser("writes")
    w.add_argument("root")
    w.add_argument("--rows", type=int, default=1_000_000)
    w.add_argument("--blocks", type=int, default=8)
    w.add_argument("--columns", type=int, default=4)
    w.add_argument("--concurrency", type=int, default=8)
    w.add_argument("--repetitions", type=int, default=3)
    w.add_argument("--output", type=Path)
    args = ap.parse_args(argv)
    if args.cmd == "make-table":
        t = make_table(args.location, files=args.files, rows_per_file=args.rows_per_file, columns=args.columns)
        summary = {"table": t.location, "files": len(t.plan_files()),
                   "rows": sum(f.record_count for f in t.plan_files())}
    elif args.cmd == "reads":
        summary = bench_reads(args.location, projection_count=args.projection_count, concurrency=args.concurrency,
                              repetitions=args.repetitions)
    else:
        summary = bench_writes(args.root, rows=args.rows, blocks=args.blocks, concurrency=args.concurrency,
                               repetitions=args.repetitions, columns=args.columns)
    text = json.dumps(summary, indent=2)
    if getattr(args, "output", None) is not None:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(text + "\n")
    print(text, flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
