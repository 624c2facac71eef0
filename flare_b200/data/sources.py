"""Pluggable sources: range reads, batching/completion policies, loaders.

Contracts follow the reference's consumption layer
(src/flare/data/pipeline/consumption/source/contracts/source.py:37-75,
batching/policies.py:15-124, execution/record_ranges.py:33,
execution/materialization.py:21-62):

* a ``SourceFactory`` plans ``WorkItem``s (record ranges of a file) and opens
  ``SourceReadSession``s that read assigned ranges;
* ``RecordRangeReadSession`` validates assigned ranges, coalesces adjacent
  ones, reads them with bounded concurrency, restores their order and keeps a
  128-entry LRU cache of materialised ranges;
* ``BatchAssembler`` cuts the record stream into fixed-size batches; the
  completion policy (carry / drop / pad / require) decides what happens to the
  incomplete tail; padded batches carry a ``BatchValidity`` (valid prefix);
* ``ParquetSourceFactory`` reads Parquet row groups with pyarrow;
  ``StandardSourceFactory`` selects a factory by name with option validation.
"""
from __future__ import annotations

import os
from collections import OrderedDict
from collections.abc import Callable, Iterable, Iterator, Mapping, Sequence
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from enum import Enum
from typing import Any, Protocol

import numpy as np

try:
    import pyarrow as pa
    import pyarrow.parquet as pq
except ImportError:  # pragma: no cover
    pa = pq = None


# ------------------------------------------------------------------ ranges
@dataclass(frozen=True, order=True)
class RecordRange:
    path: str
    start: int
    stop: int

    def __post_init__(self) -> None:
        if self.start < 0 or self.stop < self.start:
            raise ValueError(f"invalid record range [{self.start}, {self.stop})")

    @property
    def rows(self) -> int:
        return self.stop - self.start


@dataclass(frozen=True)
class WorkItem:
    item_id: int
    ranges: tuple[RecordRange, ...]

    @property
    def rows(self) -> int:
        return sum(r.rows for r in self.ranges)


def coalesce_source_ranges(ranges: Sequence[RecordRange]) -> list[RecordRange]:
    """Merge adjacent / overlapping ranges of the same file (order by file, start)."""
    out: list[RecordRange] = []
    for r in sorted(ranges):
        if out and out[-1].path == r.path and r.start <= out[-1].stop:
            out[-1] = RecordRange(r.path, out[-1].start, max(out[-1].stop, r.stop))
        else:
            out.append(r)
    return out


class SourceReadSession(Protocol):
    def read(self, item: WorkItem) -> Any: ...

    def close(self) -> None: ...


class SourceFactory(Protocol):
    def plan(self) -> list[WorkItem]: ...

    def create_session(self) -> SourceReadSession: ...


class RecordRangeReadSession:
    """Reads work items range by range with bounded concurrency and an LRU cache."""

    def __init__(self, read_range: Callable[[RecordRange], Any], concat: Callable[[list[Any]], Any], *,
                 max_concurrency: int = 4, cache_entries: int = 128, valid_paths: set[str] | None = None):
        self._read_range = read_range
        self._concat = concat
        self._pool = ThreadPoolExecutor(max_workers=max(1, max_concurrency))
        self._cache: OrderedDict[RecordRange, Any] = OrderedDict()
        self._cache_entries = cache_entries
        self._valid = valid_paths
        self.reads = 0

    def _get(self, r: RecordRange):
        if r in self._cache:
            self._cache.move_to_end(r)
            return self._cache[r]
        data = self._read_range(r)
        self.reads += 1
        self._cache[r] = data
        if len(self._cache) > self._cache_entries:
            self._cache.popitem(last=False)
        return data

    def read(self, item: WorkItem):
        for r in item.ranges:
            if self._valid is not None and r.path not in self._valid:
                raise ValueError(f"work item {item.item_id} references an unassigned file {r.path}")
        merged = coalesce_source_ranges(item.ranges)
        parts = list(self._pool.map(self._get, merged))  # map() restores the input order
        return self._concat(parts)

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        self._cache.clear()


# ----------------------------------------------------------------- parquet
class ParquetSourceFactory:
    """Work items = row groups (optionally split into ``rows_per_item`` ranges)."""

    def __init__(self, paths: Sequence[str], *, columns: Sequence[str] | None = None, rows_per_item: int | None = None,
                 max_concurrency: int = 4):
        if pq is None:
            raise RuntimeError("pyarrow is required for Parquet sources")
        self.paths = [str(p) for p in paths]
        self.columns = list(columns) if columns else None
        self.rows_per_item = rows_per_item
        self.max_concurrency = max_concurrency
        self._meta = {p: pq.ParquetFile(p).metadata for p in self.paths}

    def plan(self) -> list[WorkItem]:
        items, k = [], 0
        for p in self.paths:
            md = self._meta[p]
            start = 0
            for g in range(md.num_row_groups):
                n = md.row_group(g).num_rows
                step = self.rows_per_item or n
                for s in range(start, start + n, step):
                    items.append(WorkItem(k, (RecordRange(p, s, min(s + step, start + n)),)))
                    k += 1
                start += n
        return items

    def _read_range(self, r: RecordRange):
        f = pq.ParquetFile(r.path)
        md = f.metadata
        groups, first, acc = [], None, 0
        for g in range(md.num_row_groups):
            n = md.row_group(g).num_rows
            if acc + n > r.start and acc < r.stop:
                groups.append(g)
                if first is None:
                    first = acc
            acc += n
        t = f.read_row_groups(groups, columns=self.columns)
        return t.slice(r.start - first, r.rows)

    def create_session(self) -> RecordRangeReadSession:
        return RecordRangeReadSession(self._read_range, lambda parts: pa.concat_tables(parts),
                                      max_concurrency=self.max_concurrency, valid_paths=set(self.paths))


class StandardSourceFactory:
    """Factory selection by name with option validation."""

    KINDS = ("parquet", "files", "iceberg")

    @staticmethod
    def create(kind: str, options: Mapping[str, Any]):
        if kind not in StandardSourceFactory.KINDS:
            raise ValueError(f"unsupported source kind {kind!r}; expected one of {StandardSourceFactory.KINDS}")
        opts = dict(options)
        if kind == "iceberg":
            from .iceberg import IcebergSourceFactory

            table = opts.pop("table", None)
            if not table:
                raise ValueError("source option 'table' is required for iceberg")
            allowed = {"mode", "snapshot_id", "after_snapshot_id", "columns", "rows_per_item", "max_concurrency",
                       "cache_bytes", "cache_dir"}
            unknown = set(opts) - allowed
            if unknown:
                raise ValueError(f"unknown source options {sorted(unknown)}")
            cache_bytes, cache_dir = opts.pop("cache_bytes", None), opts.pop("cache_dir", None)
            if cache_bytes is not None:  # data files on an object store, read through a node-local cache
                from .file_cache import LocalFileCache

                opts["cache"] = LocalFileCache(int(cache_bytes), cache_dir)
            return IcebergSourceFactory(table, **opts)
        paths = opts.pop("paths", None)
        if not paths:
            raise ValueError("source option 'paths' is required")
        if isinstance(paths, str):
            paths = sorted(os.path.join(paths, f) for f in os.listdir(paths) if f.endswith(".parquet")) \
                if os.path.isdir(paths) else [paths]
        allowed = {"columns", "rows_per_item", "max_concurrency"}
        unknown = set(opts) - allowed
        if unknown:
            raise ValueError(f"unknown source options {sorted(unknown)}")
        return ParquetSourceFactory(paths, **opts)


# ---------------------------------------------------------------- batching
class CompletionPolicy(str, Enum):
    CARRY = "carry"
    DROP = "drop"
    PAD = "pad"
    REQUIRE = "require"

    @classmethod
    def from_value(cls, value) -> "CompletionPolicy":
        if isinstance(value, cls):
            return value
        v = str(value).lower()
        aliases = {"drop_remainder": "drop", "exact_aligned": "require"}
        v = aliases.get(v, v)
        try:
            return cls(v)
        except ValueError as exc:
            raise ValueError(f"Unknown completion policy {value!r}") from exc


@dataclass(frozen=True)
class BatchValidity:
    valid_count: int
    batch_size: int

    def __post_init__(self) -> None:
        if not 0 <= self.valid_count <= self.batch_size:
            raise ValueError("valid_count must be within [0, batch_size]")

    @property
    def is_padded(self) -> bool:
        return self.valid_count < self.batch_size


@dataclass
class AssembledBatch:
    data: Any
    validity: BatchValidity


class BatchAssembler:
    """Fixed-size batches from a stream of record chunks (numpy dict or Arrow tables)."""

    def __init__(self, batch_size: int, policy: str | CompletionPolicy = "carry"):
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        self.batch_size = batch_size
        self.policy = CompletionPolicy.from_value(policy)
        self._pending: list[Any] = []
        self._pending_rows = 0
        self.discarded_rows = 0

    @staticmethod
    def _rows(x) -> int:
        return x.num_rows if pa is not None and isinstance(x, pa.Table) else len(next(iter(x.values())))

    @staticmethod
    def _slice(x, a, b):
        if pa is not None and isinstance(x, pa.Table):
            return x.slice(a, b - a)
        return {k: v[a:b] for k, v in x.items()}

    @staticmethod
    def _concat(parts):
        if pa is not None and isinstance(parts[0], pa.Table):
            return pa.concat_tables(parts)
        return {k: np.concatenate([p[k] for p in parts]) for k in parts[0]}

    def push(self, chunk) -> list[AssembledBatch]:
        out = []
        self._pending.append(chunk)
        self._pending_rows += self._rows(chunk)
        while self._pending_rows >= self.batch_size:
            merged = self._concat(self._pending)
            n = self._rows(merged)
            out.append(AssembledBatch(self._slice(merged, 0, self.batch_size),
                                      BatchValidity(self.batch_size, self.batch_size)))
            rest = self._slice(merged, self.batch_size, n)
            self._pending = [rest] if n > self.batch_size else []
            self._pending_rows = n - self.batch_size
        return out

    def finish(self) -> list[AssembledBatch]:
        """Apply the completion policy to the tail."""
        if self._pending_rows == 0:
            return []
        if self.policy is CompletionPolicy.REQUIRE:
            raise ValueError(f"incomplete batch under require policy: rows={self._pending_rows} "
                             f"batch_size={self.batch_size}")
        if self.policy is CompletionPolicy.PAD:
            merged = self._concat(self._pending)
            valid = self._pending_rows
            if pa is not None and isinstance(merged, pa.Table):
                idx = np.concatenate([np.arange(valid), np.zeros(self.batch_size - valid, dtype=np.int64)])
                padded = merged.take(pa.array(idx))
            else:
                padded = {k: np.concatenate([v, np.zeros((self.batch_size - valid,) + v.shape[1:], v.dtype)])
                          for k, v in merged.items()}
            self._pending, self._pending_rows = [], 0
            return [AssembledBatch(padded, BatchValidity(valid, self.batch_size))]
        # carry (end of stream) and drop discard the tail
        self.discarded_rows += self._pending_rows
        self._pending, self._pending_rows = [], 0
        return []


def stream_batches(factory: SourceFactory, batch_size: int, *, policy: str = "carry",
                   items: Iterable[WorkItem] | None = None) -> Iterator[AssembledBatch]:
    """Read work items in order and yield assembled fixed-size batches."""
    session = factory.create_session()
    asm = BatchAssembler(batch_size, policy)
    try:
        for item in (items if items is not None else factory.plan()):
            yield from asm.push(session.read(item))
        yield from asm.finish()
    finally:
        session.close()


class StreamingBatchReader:
    """Keeps one batch assembler alive while source loaders come and go; resumable without payload.

    ``append_fragment(table, source_range)`` returns the full batches the fragment completes;
    ``finish_loader()`` ends one loader without flushing (rows carry into the next loader's
    fragments); ``finalize()`` applies the completion policy to the tail.  ``checkpoint_state()``
    holds no rows: it names the source ranges whose rows are still pending and how many leading
    rows of the first one were already emitted, so a restored reader re-reads exactly those rows
    (``replay_ranges``) before continuing.  Reference behaviour:
    src/flare/data/pipeline/consumption/source/batching/stream_reader.py:25-117.
    """

    def __init__(self, *, batch_size: int, completion_policy: str = "carry", validity_field: str | None = None):
        if validity_field is not None and (not validity_field or validity_field.strip() != validity_field):
            raise ValueError("validity_field must be a non-empty canonical string")
        self._asm = BatchAssembler(batch_size, completion_policy)
        self._validity_field = validity_field
        self._frags: list[list] = []  # [source_range, rows] of fragments with rows still pending
        self._replay: list[tuple[Any, int]] = []

    @property
    def pending_rows(self) -> int:
        return self._asm._pending_rows

    @property
    def replay_ranges(self) -> tuple[tuple[Any, int], ...]:
        """(source range, rows of it to skip) to re-read after a restore."""
        return tuple(self._replay)

    def _with_validity(self, ab: AssembledBatch):
        if self._validity_field is None:
            return ab.data
        if pa is not None and isinstance(ab.data, pa.Table):
            meta = dict(ab.data.schema.metadata or {})
            meta[self._validity_field.encode()] = str(ab.validity.valid_count).encode()
            return ab.data.replace_schema_metadata(meta)
        return {**ab.data, self._validity_field: ab.validity.valid_count}

    def _trim(self) -> None:
        """Keep only the fragments that still hold pending rows (the newest ones)."""
        left, keep = self.pending_rows, []
        for rng, rows in reversed(self._frags):
            if left <= 0:
                break
            keep.append([rng, rows])
            left -= rows
        self._frags = list(reversed(keep))

    def append_fragment(self, fragment, source_range=None) -> tuple:
        rows = fragment.num_rows if hasattr(fragment, "num_rows") else len(next(iter(fragment.values())))
        self._frags.append([source_range, rows])
        out = tuple(self._with_validity(ab) for ab in self._asm.push(fragment))
        self._trim()
        return out

    def append_loader(self, loader) -> Iterator:
        for item in loader:
            frag, rng = item if isinstance(item, tuple) else (item, None)
            yield from self.append_fragment(frag, rng)

    def finish_loader(self) -> tuple:
        return ()

    def finalize(self) -> tuple:
        out = tuple(self._with_validity(ab) for ab in self._asm.finish())
        self._frags = []
        return out

    def checkpoint_state(self) -> dict:
        pending, spans = self.pending_rows, []
        total = sum(r for _, r in self._frags)
        skip = total - pending  # rows of the first kept fragment already emitted
        for i, (rng, rows) in enumerate(self._frags):
            spans.append([rng, skip if i == 0 else 0])
        return {"pending_rows": pending, "replay": spans}

    def restore_state(self, state: Mapping[str, Any]) -> None:
        if self.pending_rows:
            raise RuntimeError("restore into a fresh reader")
        self._replay = [(rng, int(skip)) for rng, skip in state.get("replay", [])]


class ParquetRangeBatchLoader:
    """Standalone loader: static Parquet ranges of one shard -> fixed-size batches -> a caller's transform.

    ``dataset_path`` is a file or a directory of ``*.parquet`` files; ``projection`` the columns to
    read; work items (row-group ranges) are dealt to shards (item k to shard k % shard_count); every
    epoch reads this shard's items in order and yields ``batch_transformer(table)`` for each batch of
    ``batch_size`` rows, the last one padded with a validity prefix (``policy="pad"``; ``"drop"`` drops
    it, ``"carry"`` carries rows into the next epoch's first batch).  Reference behaviour:
    src/flare/data/pipeline/consumption/dataloader/parquet.py:11-90 (same arguments).
    """

    def __init__(self, *, dataset_path: str, projection: Sequence[str], batch_size: int,
                 batch_transformer: Callable[[Any], Any], shard_index: int = 0, shard_count: int = 1,
                 num_epochs: int = 1, policy: str = "pad", rows_per_item: int | None = None):
        if not isinstance(dataset_path, str) or not dataset_path:
            raise ValueError("dataset_path must be a non-empty string")
        if not projection:
            raise ValueError("projection must not be empty")
        if isinstance(batch_size, bool) or not isinstance(batch_size, int) or batch_size <= 0:
            raise ValueError("batch_size must be a positive integer")
        if not callable(batch_transformer):
            raise TypeError("batch_transformer must be callable")
        for v, n in ((shard_index, "shard_index"), (shard_count, "shard_count"), (num_epochs, "num_epochs")):
            if isinstance(v, bool) or not isinstance(v, int) or v < 0:
                raise ValueError(f"{n} must be a non-negative integer")
        if shard_count < 1 or shard_index >= shard_count:
            raise ValueError("shard_index must be in [0, shard_count)")
        if os.path.isdir(dataset_path):
            paths = sorted(os.path.join(dataset_path, f) for f in os.listdir(dataset_path) if f.endswith(".parquet"))
        else:
            paths = [dataset_path]
        if not paths:
            raise ValueError(f"no Parquet files under {dataset_path}")
        self.factory = ParquetSourceFactory(paths, columns=list(projection), rows_per_item=rows_per_item)
        self.items = [it for k, it in enumerate(self.factory.plan()) if k % shard_count == shard_index]
        self.batch_size, self.transform, self.num_epochs, self.policy = batch_size, batch_transformer, num_epochs, policy
        self.last_validity: BatchValidity | None = None

    def __iter__(self) -> Iterator[Any]:
        session = self.factory.create_session()
        asm = BatchAssembler(self.batch_size, self.policy)
        try:
            for epoch in range(self.num_epochs):
                for item in self.items:
                    for ab in asm.push(session.read(item)):
                        self.last_validity = ab.validity
                        yield self.transform(ab.data)
                if self.policy != "carry" or epoch == self.num_epochs - 1:
                    for ab in asm.finish():
                        self.last_validity = ab.validity  # a padded batch's valid prefix
                        yield self.transform(ab.data)
        finally:
            session.close()


__all__ = [
    "AssembledBatch", "BatchAssembler", "BatchValidity", "CompletionPolicy", "ParquetRangeBatchLoader",
    "ParquetSourceFactory", "RecordRange", "StreamingBatchReader",
    "RecordRangeReadSession", "SourceFactory", "SourceReadSession", "StandardSourceFactory", "WorkItem",
    "coalesce_source_ranges", "stream_batches",
]
