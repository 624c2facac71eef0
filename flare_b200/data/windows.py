"""Producer windows: cut a record file into fixed-size window files for continuous-ingestion runs.

``write_stream_windows(source, target, rows_per_window=, windows=, start_window=)`` reads the first
``rows_per_window * (start_window + windows)`` records of ``source`` (plain, gzip or zstd, the record
files the feature pipeline reads) and writes windows ``start_window .. start_window + windows - 1`` as
``target/part-<window>.txt`` (or ``.zst``): each file holds its window's records, one per line,
published atomically (written and synced under a private dot-name the pipeline's lister skips, then
hard-linked to its final name, which fails if that window exists), and read back to check its record
count.  A window is what an upstream producer drops per period, so
a run of the pipeline over a growing ``target`` directory (``data.pipeline``, publication windows and
resume state) can be driven locally, window by window.

    python -m flare_b200.data.windows SOURCE TARGET --rows-per-window 64 --windows 3 [--start-window 0]
        [--compression plain|zstd]

Reference counterpart: tools/validation/generate_stream_windows.py (fixed-size producer windows for
live ingestion validation).
"""
from __future__ import annotations

import argparse
import os
from pathlib import Path

import pyarrow as pa

from .pipeline import _open_text as open_record_text


def read_records(source: str | os.PathLike, count: int) -> list[str]:
    """The first ``count`` non-empty records of ``source``; fewer records or an empty one is an error."""
    out: list[str] = []
    with open_record_text(str(source)) as f:
        for line in f:
            rec = line.rstrip("\r\n")
            if not rec:
                raise ValueError(f"{source}: empty record at line {len(out) + 1}")
            out.append(rec)
            if len(out) == count:
                break
    if len(out) != count:
        raise ValueError(f"{source} has {len(out)} records, {count} needed")
    return out


def _decode(path: Path) -> bytes:
    if path.suffix == ".zst":
        with pa.input_stream(str(path), compression="zstd") as s:
            return s.read()
    return path.read_bytes()


def write_stream_windows(source: str | os.PathLike, target: str | os.PathLike, *, rows_per_window: int,
                         windows: int, start_window: int = 0, compression: str = "plain") -> list[Path]:
    if rows_per_window <= 0 or windows <= 0 or start_window < 0:
        raise ValueError("rows_per_window and windows must be positive, start_window non-negative")
    if compression not in ("plain", "zstd"):
        raise ValueError(f"compression must be 'plain' or 'zstd', got {compression!r}")
    records = read_records(source, rows_per_window * (start_window + windows))
    tdir = Path(target)
    tdir.mkdir(parents=True, exist_ok=True)
    written = []
    for w in range(start_window, start_window + windows):
        chunk = records[w * rows_per_window:(w + 1) * rows_per_window]
        body = ("\n".join(chunk) + "\n").encode("utf-8")
        path = tdir / f"part-{w:05d}{'.zst' if compression == 'zstd' else '.txt'}"
        if path.exists():
            raise FileExistsError(path)
        data = pa.compress(body, codec="zstd", asbytes=True) if compression == "zstd" else body
        scratch = tdir / f".{path.name}.{os.getpid()}.partial"
        try:
            with open(scratch, "wb") as f:
                f.write(data)
                f.flush()
                os.fsync(f.fileno())
            os.link(scratch, path)  # fails if another producer published this window meanwhile
        finally:
            scratch.unlink(missing_ok=True)
        if len(_decode(path).splitlines()) != rows_per_window:
            raise AssertionError(f"{path} does not decode to {rows_per_window} records")
        written.append(path)
    return written


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="cut a record file into fixed-size producer windows")
    ap.add_argument("source")
    ap.add_argument("target")
    ap.add_argument("--rows-per-window", type=int, default=64)
    ap.add_argument("--windows", type=int, default=3)
    ap.add_argument("--start-window", type=int, default=0)
    ap.add_argument("--compression", choices=("plain", "zstd"), default="plain")
    a = ap.parse_args(argv)
    paths = write_stream_windows(a.source, a.target, rows_per_window=a.rows_per_window, windows=a.windows,
                                 start_window=a.start_window, compression=a.compression)
    print(f"windows={len(paths)} rows_per_window={a.rows_per_window} compression={a.compression}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["read_records", "write_stream_windows"]
