"""Node-local cache of immutable remote data files (Iceberg data files on an object store).

The Parquet readers of this package read local files (memory-mapped range reads).  A table whose
data files live on an object store is read through ``LocalFileCache``: ``local_path(uri, identity)``
returns a local copy of the object, downloading it once per node.

* Entries are named by a digest of ``identity`` and the URI.  An Iceberg data file never changes
  after its commit, so its size (or any revision string) plus its path identifies the bytes.
* A download streams the object into a private ``*.partial`` file and renames it into place, under a
  per-entry ``flock``, so concurrent readers of one node (threads or processes) download an entry
  once and never see a partial file.
* Using an entry refreshes its modification time; after a download the least recently used entries
  are removed until the cache fits ``max_bytes`` again.  The entry just returned and every entry this
  cache object returned since its last ``release()`` (a scan's files, which its readers open later)
  are never removed, so a scan larger than the budget is still served; other processes sharing the
  directory may remove them, so size one directory for the concurrent scans of a node.  A file that
  is open stays readable after its entry is removed (POSIX unlink semantics).

Reference behaviour: src/flare/data/connectors/adapters/parquet/local_cache.py (bounded node-local
cache of immutable Iceberg Parquet files with per-entry locks and LRU eviction).
"""
from __future__ import annotations

import fcntl
import hashlib
import os
import threading
from pathlib import Path

from ..io.objectstore import ObjectStoreIO

_CHUNK = 8 << 20


class LocalFileCache:
    def __init__(self, max_bytes: int, directory: str | os.PathLike | None = None, *,
                 io: ObjectStoreIO | None = None):
        if type(max_bytes) is not int or max_bytes <= 0:
            raise ValueError("the cache size must be a positive number of bytes")
        self.max_bytes = max_bytes
        self.io = io or ObjectStoreIO()
        self.directory = Path(directory) if directory is not None else \
            Path("/tmp") / f"flare-b200-file-cache-{os.getuid()}"
        self.directory.mkdir(mode=0o700, parents=True, exist_ok=True)
        if self.directory.stat().st_uid != os.getuid():
            raise PermissionError(f"{self.directory} belongs to another user")
        self.stats = {"hits": 0, "downloads": 0, "evictions": 0, "bytes_downloaded": 0}
        self._lock = threading.Lock()
        self._pinned: set[Path] = set()

    def release(self) -> None:
        """Let eviction remove the entries this object returned so far."""
        with self._lock:
            self._pinned.clear()

    def _entry(self, uri: str, identity: str) -> str:
        if not uri or not identity:
            raise ValueError("a cache entry needs a URI and an identity")
        return hashlib.sha256(f"{identity}\0{uri}".encode("utf-8")).hexdigest()

    def _count(self, key: str, n: int = 1) -> None:
        with self._lock:
            self.stats[key] += n

    def local_path(self, uri: str, identity: str) -> str:
        """A local file holding the bytes of ``uri`` (downloaded on first use on this node)."""
        digest = self._entry(str(uri), str(identity))
        target = self.directory / f"{digest}.data"
        downloaded = False
        with open(self.directory / f"{digest}.lock", "a+b") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                if target.is_file():
                    self._count("hits")
                else:
                    for stale in self.directory.glob(f"{digest}.*.partial"):  # left by a crashed download
                        stale.unlink(missing_ok=True)
                    partial = self.directory / f"{digest}.{os.getpid()}.{threading.get_ident()}.partial"
                    fs, inner, _ = self.io.resolve(uri)

                    def copy() -> int:
                        n = 0
                        with fs.open_input_stream(inner) as src, open(partial, "wb") as dst:
                            while chunk := src.read(_CHUNK):
                                dst.write(chunk)
                                n += len(chunk)
                        return n

                    try:
                        n = self.io._retry(f"download {uri}", copy)
                        os.replace(partial, target)
                    finally:
                        partial.unlink(missing_ok=True)
                    downloaded = True
                    self._count("downloads")
                    self._count("bytes_downloaded", n)
                os.utime(target, None)
                with self._lock:
                    self._pinned.add(target)
            finally:
                fcntl.flock(lock, fcntl.LOCK_UN)
        if downloaded:
            self._evict(keep=target)
        return str(target)

    def cached_bytes(self) -> int:
        return sum(p.stat().st_size for p in self.directory.glob("*.data"))

    def _evict(self, *, keep: Path) -> None:
        """Remove the least recently used entries until the cache fits (never ``keep``)."""
        with open(self.directory / ".evict.lock", "a+b") as glock:
            fcntl.flock(glock, fcntl.LOCK_EX)
            try:
                entries = []
                for p in self.directory.glob("*.data"):
                    try:
                        st = p.stat()
                    except FileNotFoundError:
                        continue
                    entries.append((st.st_mtime_ns, st.st_size, p))
                total = sum(size for _, size, _ in entries)
                for _, size, p in sorted(entries):
                    if total <= self.max_bytes:
                        break
                    with self._lock:
                        pinned = p == keep or p in self._pinned
                    if pinned:
                        continue
                    with open(p.with_suffix(".lock"), "a+b") as lock:  # not while a reader downloads it
                        fcntl.flock(lock, fcntl.LOCK_EX)
                        try:
                            p.unlink(missing_ok=True)
                        finally:
                            fcntl.flock(lock, fcntl.LOCK_UN)
                    total -= size
                    self._count("evictions")
            finally:
                fcntl.flock(glock, fcntl.LOCK_UN)


__all__ = ["LocalFileCache"]
