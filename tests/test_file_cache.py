"""Node-local cache of remote data files: an Iceberg table on an (in-memory) object store is scanned
through the cache, files download once, least recently used entries go when the budget is exceeded,
and the entries a scan still needs stay (CPU)."""
from datetime import datetime

import pytest

pa = pytest.importorskip("pyarrow")
pafs = pytest.importorskip("pyarrow.fs")

from flare_b200.data.file_cache import LocalFileCache  # noqa: E402
from flare_b200.data.iceberg import IcebergSink, IcebergSourceFactory, IcebergTable  # noqa: E402
from flare_b200.data.reader import BatchReader  # noqa: E402
from flare_b200.io.objectstore import ObjectStoreIO  # noqa: E402


def _remote_table():
    mock = pafs._MockFileSystem(datetime(2024, 1, 1))
    store = ObjectStoreIO(filesystems={"s3": mock})
    for d in ("bucket/t/metadata", "bucket/t/data"):  # an object store needs no directories; the mock does
        mock.create_dir(d)
    data = pa.table({"x": list(range(300))})
    t = IcebergTable.create("s3://bucket/t", data.schema, io=store)
    IcebergSink(t).append([data.slice(0, 100), data.slice(100, 100), data.slice(200, 100)])
    return t.refresh(), store


def test_remote_iceberg_scan_through_the_cache(tmp_path):
    t, store = _remote_table()
    with pytest.raises(ValueError, match="local cache"):
        IcebergSourceFactory(t)
    cache = LocalFileCache(1 << 30, tmp_path / "cache", io=store)
    fac = IcebergSourceFactory(t, cache=cache)
    rows = [v for b, val in BatchReader(fac, 64) for v in b.column("x").to_pylist()[:val.valid_count]]
    assert sorted(rows) == list(range(300))
    assert cache.stats["downloads"] == 3 and cache.stats["hits"] == 0
    IcebergSourceFactory(t, cache=cache)  # the same files again: no download
    assert cache.stats["downloads"] == 3 and cache.stats["hits"] == 3


def test_budget_evicts_least_recently_used_but_not_pinned_entries(tmp_path):
    t, store = _remote_table()
    sizes = [f.file_size_in_bytes for f in t.plan_files()]
    budget = 2 * max(sizes) + 1  # room for two files
    scan = LocalFileCache(budget, tmp_path / "c", io=store)
    paths = [scan.local_path(f.path, f"size={f.file_size_in_bytes}") for f in t.plan_files()]
    assert scan.stats["evictions"] == 0 and scan.cached_bytes() > budget  # one scan's files are pinned
    scan.release()
    other = LocalFileCache(budget, tmp_path / "c", io=store)
    f0 = t.plan_files()[0]
    other.local_path(f0.path, f"size={f0.file_size_in_bytes}")  # hit: refreshes file 0
    assert other.stats["hits"] == 1
    import os
    # file 1, then file 2 are the least recently used (explicit times: the file clock is coarser than
    # the few microseconds between these calls)
    os.utime(paths[1], ns=(1, 1))
    os.utime(paths[2], ns=(2, 2))
    extra = LocalFileCache(budget, tmp_path / "c", io=store)
    extra.local_path(f0.path, "size=changed")  # another revision of file 0: a download, then eviction
    assert not os.path.exists(paths[1]) and os.path.exists(paths[0])
    assert extra.cached_bytes() <= budget
    with pytest.raises(ValueError):
        LocalFileCache(0, tmp_path / "d")
