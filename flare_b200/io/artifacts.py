"""Crash-safe small artifacts (manifests, leases, audits) on a local or mounted filesystem.

The primitive is :func:`publish_bytes`: the payload is written in full to a
private sibling file, made durable, and only then given the artifact's name,
so a reader sees either the previous artifact or the new one, never a torn
write.  Two ways to give it the name:

* ``replace`` (default): the new artifact supersedes any old one;
* ``create``: the name is taken only if nobody holds it yet (a lease or a
  "first writer wins" marker); a holder makes the call raise
  ``FileExistsError``.

JSON helpers sit on top.  Reference behaviour (what the pipeline's leases and
manifests rely on): src/flare/io/artifacts.py:14-45.
"""
from __future__ import annotations

import itertools
import json
import os
import secrets
from pathlib import Path
from typing import Any

_SEQ = itertools.count()


def companion_file(path: Path, suffix: str) -> Path:
    """The file beside ``path`` whose name is ``path``'s name followed by ``suffix``."""
    path = Path(path)
    return path.parent / f"{path.name}{suffix}"


def _private_sibling(path: Path) -> Path:
    # unique per process, call and random token: concurrent writers never share a scratch file
    return path.parent / f".{path.name}.{os.getpid()}-{next(_SEQ)}-{secrets.token_hex(4)}.partial"


def _sync_directory(directory: Path) -> None:
    """Make a rename / link inside ``directory`` durable (no-op where directories cannot be opened)."""
    try:
        fd = os.open(directory, os.O_RDONLY | getattr(os, "O_DIRECTORY", 0))
    except OSError:
        return
    try:
        os.fsync(fd)
    except OSError:
        pass
    finally:
        os.close(fd)


def publish_bytes(path: Path | str, payload: bytes, *, mode: str = "replace") -> Path:
    """Durably give ``payload`` the name ``path`` (``mode``: ``"replace"`` or ``"create"``)."""
    if mode not in ("replace", "create"):
        raise ValueError(f"unknown publish mode {mode!r}")
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    scratch = _private_sibling(path)
    fd = os.open(scratch, os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o644)
    try:
        view = memoryview(payload)
        while view:
            view = view[os.write(fd, view):]
        os.fsync(fd)
    finally:
        os.close(fd)
    try:
        if mode == "create":
            os.link(scratch, path)  # atomic "create if absent": raises FileExistsError for a holder
        else:
            os.replace(scratch, path)
        _sync_directory(path.parent)
    finally:
        if scratch.exists():
            scratch.unlink()
    return path


def write_json(path: Path | str, value: Any, *, exclusive: bool = False) -> None:
    """Publish ``value`` as UTF-8 JSON (keys sorted, one trailing newline); ``exclusive``: create only."""
    text = json.dumps(value, indent=2, ensure_ascii=False, sort_keys=True) + "\n"
    publish_bytes(path, text.encode("utf-8"), mode="create" if exclusive else "replace")


def read_json(path: Path | str) -> Any:
    with open(path, "rb") as f:
        return json.loads(f.read().decode("utf-8"))


__all__ = ["companion_file", "publish_bytes", "read_json", "write_json"]
