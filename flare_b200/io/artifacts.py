"""Durable JSON artifacts: write to a temp file, fsync, then rename (or hard-link when exclusive).

A reader never sees a half-written file; ``exclusive=True`` fails if the
artifact already exists (first writer wins).  Reference behaviour:
src/flare/io/artifacts.py:14-45.
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path
from typing import Any


def companion_file(path: Path, suffix: str) -> Path:
    return path.with_suffix(path.suffix + suffix)


def write_json(path: Path | str, value: Any, *, exclusive: bool = False) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
    tmp_path = Path(tmp)
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as f:
            json.dump(value, f, indent=2, ensure_ascii=False, sort_keys=True)
            f.write("\n")
            f.flush()
            os.fsync(f.fileno())
        if exclusive:
            os.link(tmp_path, path)   # FileExistsError when the artifact exists
        else:
            os.replace(tmp_path, path)
        dfd = os.open(path.parent, os.O_RDONLY | os.O_DIRECTORY)
        try:
            os.fsync(dfd)
        finally:
            os.close(dfd)
    finally:
        tmp_path.unlink(missing_ok=True)


def read_json(path: Path | str) -> Any:
    return json.loads(Path(path).read_text(encoding="utf-8"))


__all__ = ["companion_file", "read_json", "write_json"]
