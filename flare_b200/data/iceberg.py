"""Apache Iceberg tables (format v2) on a filesystem, without an Iceberg client library.

Layout (the file-system catalog of the Iceberg specification): a table at
``location`` keeps its data files under ``data/`` and its metadata under
``metadata/``: ``v<N>.metadata.json`` (the table metadata: schemas with
field ids, the unpartitioned spec, snapshots, refs, logs),
``version-hint.text`` (the current N), per snapshot a manifest list
``snap-<id>-<uuid>.avro`` and per commit a manifest ``<uuid>-m0.avro`` (Avro
object containers, ``data/avro.py``).  Manifest entries carry status
(0 existing, 1 added, 2 deleted), snapshot id and sequence numbers (null in
an added entry: inherited from its manifest, as v2 prescribes) and the data
file (path, format, record count, size).  The Avro field ids are the
specification's.

* ``IcebergTable.create / load``; ``schema()``, ``snapshots()``,
  ``current_snapshot()``.
* Scans: ``plan_files(snapshot_id)`` (pinned snapshot: every live data file,
  manifests read one at a time), ``appended_files(after, upto)`` (continuous
  append: the files added by the append snapshots after ``after``).
* Commits: ``append(files, commit_id=...)`` writes a manifest, a manifest
  list (the parent's manifests plus the new one) and ``v<N+1>`` with an
  atomic create-if-absent on local storage (a concurrent committer that wins
  makes this one re-read the table and retry); ``commit_id`` goes into the
  snapshot summary, so ``append`` is idempotent and ``find_commit`` tells a
  restarted writer whether its commit landed; ``orphan_files()`` lists data
  files no snapshot references (left by a writer that died before
  committing).
* ``IcebergSink`` writes Arrow tables as Parquet data files (Iceberg field
  ids in the Parquet schema) and commits them; ``IcebergSourceFactory`` plans
  the files of a snapshot (or the appends after a cursor snapshot) as work
  items for ``BatchReader`` / ``stream_batches``.

Reference behaviour: src/flare/data/connectors/adapters/iceberg/ (source.py
planner and scan :154,450, manifest_stream.py:40 bounded traversal, sink.py:65
snapshot publisher, recovery.py:22, modes.py:7,16 ContinuousAppend /
PinnedSnapshot).  Object stores without an atomic create are written with
check-then-put (one committer per table there).
"""
from __future__ import annotations

import json
import os
import random
import time
import uuid
from collections.abc import Iterable, Iterator, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import pyarrow as pa
import pyarrow.parquet as pq

from . import avro
from .sources import ParquetSourceFactory, RecordRangeReadSession, WorkItem

FORMAT_VERSION = 2
COMMIT_ID = "flare.commit-id"
STATUS_EXISTING, STATUS_ADDED, STATUS_DELETED = 0, 1, 2

# ------------------------------------------------------------- Avro schemas of the specification
_DATA_FILE = {"type": "record", "name": "r2", "fields": [
    {"name": "content", "type": "int", "field-id": 134},
    {"name": "file_path", "type": "string", "field-id": 100},
    {"name": "file_format", "type": "string", "field-id": 101},
    {"name": "partition", "type": {"type": "record", "name": "r102", "fields": []}, "field-id": 102},
    {"name": "record_count", "type": "long", "field-id": 103},
    {"name": "file_size_in_bytes", "type": "long", "field-id": 104},
]}
MANIFEST_ENTRY = {"type": "record", "name": "manifest_entry", "fields": [
    {"name": "status", "type": "int", "field-id": 0},
    {"name": "snapshot_id", "type": ["null", "long"], "default": None, "field-id": 1},
    {"name": "sequence_number", "type": ["null", "long"], "default": None, "field-id": 3},
    {"name": "file_sequence_number", "type": ["null", "long"], "default": None, "field-id": 4},
    {"name": "data_file", "type": _DATA_FILE, "field-id": 2},
]}
MANIFEST_FILE = {"type": "record", "name": "manifest_file", "fields": [
    {"name": "manifest_path", "type": "string", "field-id": 500},
    {"name": "manifest_length", "type": "long", "field-id": 501},
    {"name": "partition_spec_id", "type": "int", "field-id": 502},
    {"name": "content", "type": "int", "field-id": 517},
    {"name": "sequence_number", "type": "long", "field-id": 515},
    {"name": "min_sequence_number", "type": "long", "field-id": 516},
    {"name": "added_snapshot_id", "type": "long", "field-id": 503},
    {"name": "added_files_count", "type": "int", "field-id": 504},
    {"name": "existing_files_count", "type": "int", "field-id": 505},
    {"name": "deleted_files_count", "type": "int", "field-id": 506},
    {"name": "added_rows_count", "type": "long", "field-id": 512},
    {"name": "existing_rows_count", "type": "long", "field-id": 513},
    {"name": "deleted_rows_count", "type": "long", "field-id": 514},
]}


# ------------------------------------------------------------- schema conversion
def _iceberg_type(t: pa.DataType, next_id) -> Any:
    if pa.types.is_boolean(t):
        return "boolean"
    if pa.types.is_int8(t) or pa.types.is_int16(t) or pa.types.is_int32(t) or pa.types.is_uint8(t) \
            or pa.types.is_uint16(t):
        return "int"
    if pa.types.is_integer(t):
        return "long"
    if pa.types.is_float32(t) or pa.types.is_float16(t):
        return "float"
    if pa.types.is_float64(t):
        return "double"
    if pa.types.is_string(t) or pa.types.is_large_string(t):
        return "string"
    if pa.types.is_binary(t) or pa.types.is_large_binary(t):
        return "binary"
    if pa.types.is_date(t):
        return "date"
    if pa.types.is_timestamp(t):
        return "timestamptz" if t.tz else "timestamp"
    if pa.types.is_list(t) or pa.types.is_large_list(t):
        eid = next_id()
        return {"type": "list", "element-id": eid, "element": _iceberg_type(t.value_type, next_id),
                "element-required": False}
    if pa.types.is_struct(t):
        return {"type": "struct", "fields": [_field(t.field(i), next_id) for i in range(t.num_fields)]}
    raise ValueError(f"no Iceberg type for Arrow type {t}")


def _field(f: pa.Field, next_id) -> dict:
    fid = next_id()
    return {"id": fid, "name": f.name, "required": not f.nullable, "type": _iceberg_type(f.type, next_id)}


def iceberg_schema(schema: pa.Schema, schema_id: int = 0) -> dict:
    """Iceberg schema JSON with field ids assigned depth-first from 1."""
    counter = [0]

    def next_id():
        counter[0] += 1
        return counter[0]

    fields = [_field(f, next_id) for f in schema]
    return {"type": "struct", "schema-id": schema_id, "fields": fields, "_last_id": counter[0]}


def _with_field_ids(schema: pa.Schema, ischema: dict) -> pa.Schema:
    """Arrow schema whose fields carry the Iceberg field ids (Parquet ``field_id``)."""

    def conv(f: pa.Field, node: dict) -> pa.Field:
        t, it = f.type, node["type"]
        if isinstance(it, dict) and it["type"] == "list":
            el = pa.field("element", t.value_type, True, {b"PARQUET:field_id": str(it["element-id"]).encode()})
            t = pa.list_(el)
        elif isinstance(it, dict) and it["type"] == "struct":
            t = pa.struct([conv(t.field(i), it["fields"][i]) for i in range(t.num_fields)])
        return pa.field(f.name, t, f.nullable, {b"PARQUET:field_id": str(node["id"]).encode()})

    return pa.schema([conv(f, n) for f, n in zip(schema, ischema["fields"])])


@dataclass(frozen=True)
class DataFile:
    path: str
    record_count: int
    file_size_in_bytes: int
    snapshot_id: int | None = None
    sequence_number: int | None = None
    file_format: str = "PARQUET"


class CommitConflict(RuntimeError):
    pass


# ------------------------------------------------------------- the table
class IcebergTable:
    def __init__(self, location: str | os.PathLike, *, io=None):
        from ..io.objectstore import ObjectStoreIO

        loc = str(location).rstrip("/")
        self._local = "://" not in loc or loc.startswith("file://")
        if "://" not in loc:
            loc = str(Path(loc).absolute())
        self.location = loc
        self.io = io or ObjectStoreIO()
        self.version, self.meta = self._load_latest()

    # ---------------------------------------------------------- paths / io
    def _p(self, *parts: str) -> str:
        return "/".join([self.location, *parts])

    def _read_json(self, path: str) -> dict:
        return json.loads(self.io.read_bytes(path).decode("utf-8"))

    def _create(self, path: str, data: bytes) -> None:
        """Create ``path`` only if it does not exist (atomic on local storage)."""
        if self._local:
            from ..io.artifacts import publish_bytes

            local = path[len("file://"):] if path.startswith("file://") else path
            try:
                publish_bytes(local, data, mode="create")
            except FileExistsError as e:
                raise CommitConflict(path) from e
            return
        if self.io.exists(path):
            raise CommitConflict(path)
        self.io.write_bytes(path, data)

    def _load_latest(self) -> tuple[int, dict | None]:
        hint = self._p("metadata", "version-hint.text")
        v = 0
        if self.io.exists(hint):
            v = int(self.io.read_bytes(hint).decode().strip() or 0)
        # the hint may lag a commit that was not followed by its hint update
        while self.io.exists(self._p("metadata", f"v{v + 1}.metadata.json")):
            v += 1
        if v == 0:
            return 0, None
        return v, self._read_json(self._p("metadata", f"v{v}.metadata.json"))

    def refresh(self) -> "IcebergTable":
        self.version, self.meta = self._load_latest()
        return self

    # ---------------------------------------------------------- create / load
    @classmethod
    def create(cls, location: str | os.PathLike, schema: pa.Schema, *, properties: dict[str, str] | None = None,
               io=None, exist_ok: bool = False) -> "IcebergTable":
        t = cls(location, io=io)
        if t.meta is not None:
            if exist_ok:
                return t
            raise FileExistsError(f"an Iceberg table exists at {t.location}")
        ischema = iceberg_schema(schema)
        last_id = ischema.pop("_last_id")
        now = int(time.time() * 1000)
        meta = {
            "format-version": FORMAT_VERSION, "table-uuid": str(uuid.uuid4()), "location": t.location,
            "last-sequence-number": 0, "last-updated-ms": now, "last-column-id": last_id,
            "current-schema-id": 0, "schemas": [ischema], "default-spec-id": 0,
            "partition-specs": [{"spec-id": 0, "fields": []}], "last-partition-id": 999,
            "default-sort-order-id": 0, "sort-orders": [{"order-id": 0, "fields": []}],
            "properties": dict(properties or {}), "current-snapshot-id": -1, "refs": {}, "snapshots": [],
            "snapshot-log": [], "metadata-log": [],
        }
        t._commit_metadata(meta)
        return t

    @classmethod
    def load(cls, location: str | os.PathLike, *, io=None) -> "IcebergTable":
        t = cls(location, io=io)
        if t.meta is None:
            raise FileNotFoundError(f"no Iceberg table at {t.location}")
        return t

    def _commit_metadata(self, meta: dict) -> None:
        v = self.version + 1
        path = self._p("metadata", f"v{v}.metadata.json")
        self._create(path, (json.dumps(meta, indent=2) + "\n").encode())
        self.io.write_bytes(self._p("metadata", "version-hint.text"), str(v).encode())
        self.version, self.meta = v, meta

    # ---------------------------------------------------------- reads
    def schema(self) -> dict:
        sid = self.meta["current-schema-id"]
        return next(s for s in self.meta["schemas"] if s["schema-id"] == sid)

    def arrow_schema(self) -> pa.Schema:
        def conv(t):
            if isinstance(t, dict):
                if t["type"] == "list":
                    return pa.list_(conv(t["element"]))
                if t["type"] == "struct":
                    return pa.struct([pa.field(f["name"], conv(f["type"]), not f["required"]) for f in t["fields"]])
            return {"boolean": pa.bool_(), "int": pa.int32(), "long": pa.int64(), "float": pa.float32(),
                    "double": pa.float64(), "string": pa.string(), "binary": pa.binary(), "date": pa.date32(),
                    "timestamp": pa.timestamp("us"), "timestamptz": pa.timestamp("us", "UTC")}[t]

        return pa.schema([pa.field(f["name"], conv(f["type"]), not f["required"]) for f in self.schema()["fields"]])

    def snapshots(self) -> list[dict]:
        return list(self.meta["snapshots"]) if self.meta else []

    def snapshot(self, snapshot_id: int) -> dict:
        for s in self.snapshots():
            if s["snapshot-id"] == snapshot_id:
                return s
        raise KeyError(f"no snapshot {snapshot_id}")

    def current_snapshot(self) -> dict | None:
        sid = self.meta.get("current-snapshot-id", -1) if self.meta else -1
        return None if sid in (None, -1) else self.snapshot(sid)

    def manifests(self, snapshot: dict) -> list[dict]:
        recs, _ = avro.read_container(self.io.read_bytes(snapshot["manifest-list"]))
        return recs

    def manifest_entries(self, manifest: dict) -> Iterator[dict]:
        """Entries of one manifest with inherited sequence numbers filled in."""
        for e in avro.ContainerReader(self.io.read_bytes(manifest["manifest_path"])):
            if e["sequence_number"] is None and e["status"] == STATUS_ADDED:
                e["sequence_number"] = manifest["sequence_number"]
            if e["file_sequence_number"] is None and e["status"] == STATUS_ADDED:
                e["file_sequence_number"] = manifest["sequence_number"]
            if e["snapshot_id"] is None:
                e["snapshot_id"] = manifest["added_snapshot_id"]
            yield e

    def plan_files(self, snapshot_id: int | None = None) -> list[DataFile]:
        """Every live data file of a snapshot (default: the current one), manifests read one at a time."""
        snap = self.current_snapshot() if snapshot_id is None else self.snapshot(snapshot_id)
        if snap is None:
            return []
        out = []
        for m in self.manifests(snap):
            if m["content"] != 0:
                continue
            for e in self.manifest_entries(m):
                if e["status"] != STATUS_DELETED and e["data_file"]["content"] == 0:
                    d = e["data_file"]
                    out.append(DataFile(d["file_path"], d["record_count"], d["file_size_in_bytes"], e["snapshot_id"],
                                        e["sequence_number"], d["file_format"]))
        return out

    def ancestry(self, snapshot_id: int | None = None) -> list[dict]:
        """Snapshots from ``snapshot_id`` (default current) back to the first, newest first."""
        snap = self.current_snapshot() if snapshot_id is None else self.snapshot(snapshot_id)
        out = []
        while snap is not None:
            out.append(snap)
            parent = snap.get("parent-snapshot-id")
            snap = self.snapshot(parent) if parent is not None else None
        return out

    def appended_files(self, after_snapshot_id: int | None, upto_snapshot_id: int | None = None) -> list[DataFile]:
        """Files added by the append snapshots after ``after_snapshot_id`` up to ``upto`` (oldest first)."""
        chain = self.ancestry(upto_snapshot_id)
        ids = [s["snapshot-id"] for s in chain]
        if after_snapshot_id is not None and after_snapshot_id not in ids:
            raise ValueError(f"snapshot {after_snapshot_id} is not an ancestor of the scan's end snapshot")
        newer = []
        for s in chain:
            if s["snapshot-id"] == after_snapshot_id:
                break
            newer.append(s)
        out = []
        for s in reversed(newer):
            if s.get("summary", {}).get("operation") != "append":
                raise ValueError(f"snapshot {s['snapshot-id']} is a {s.get('summary', {}).get('operation')}; "
                                 "continuous scans follow appends only")
            for m in self.manifests(s):
                if m["added_snapshot_id"] != s["snapshot-id"]:
                    continue
                for e in self.manifest_entries(m):
                    if e["status"] == STATUS_ADDED:
                        d = e["data_file"]
                        out.append(DataFile(d["file_path"], d["record_count"], d["file_size_in_bytes"],
                                            s["snapshot-id"], e["sequence_number"], d["file_format"]))
        return out

    def find_commit(self, commit_id: str) -> dict | None:
        for s in self.snapshots():
            if s.get("summary", {}).get(COMMIT_ID) == commit_id:
                return s
        return None

    # ---------------------------------------------------------- commits
    def append(self, files: Sequence[DataFile], *, commit_id: str | None = None, attempts: int = 8) -> dict:
        """Commit ``files`` as one append snapshot (idempotent per ``commit_id``)."""
        if not files:
            raise ValueError("an append needs at least one data file")
        for attempt in range(attempts):
            self.refresh()
            if self.meta is None:
                raise FileNotFoundError(f"no Iceberg table at {self.location}")
            if commit_id is not None:
                done = self.find_commit(commit_id)
                if done is not None:
                    return done
            try:
                return self._append_once(files, commit_id)
            except CommitConflict:
                time.sleep(0.01 * (attempt + 1) * random.random())
        raise CommitConflict(f"append to {self.location} lost {attempts} races")

    def _append_once(self, files: Sequence[DataFile], commit_id: str | None) -> dict:
        meta = json.loads(json.dumps(self.meta))
        parent = self.current_snapshot()
        seq = meta["last-sequence-number"] + 1
        sid = random.getrandbits(62) + 1
        now = int(time.time() * 1000)
        tag = uuid.uuid4().hex
        entries = [{"status": STATUS_ADDED, "snapshot_id": sid, "sequence_number": None,
                    "file_sequence_number": None,
                    "data_file": {"content": 0, "file_path": f.path, "file_format": f.file_format, "partition": {},
                                  "record_count": int(f.record_count), "file_size_in_bytes": int(f.file_size_in_bytes)}}
                   for f in files]
        mpath = self._p("metadata", f"{tag}-m0.avro")
        mbytes = avro.container_bytes(MANIFEST_ENTRY, entries, metadata={
            "schema": json.dumps(self.schema()), "schema-id": str(self.schema()["schema-id"]),
            "partition-spec": "[]", "partition-spec-id": "0", "format-version": str(FORMAT_VERSION),
            "content": "data"})
        self.io.write_bytes(mpath, mbytes)
        manifests = self.manifests(parent) if parent is not None else []
        new = {"manifest_path": mpath, "manifest_length": len(mbytes), "partition_spec_id": 0, "content": 0,
               "sequence_number": seq, "min_sequence_number": seq, "added_snapshot_id": sid,
               "added_files_count": len(files), "existing_files_count": 0, "deleted_files_count": 0,
               "added_rows_count": sum(int(f.record_count) for f in files), "existing_rows_count": 0,
               "deleted_rows_count": 0}
        lpath = self._p("metadata", f"snap-{sid}-1-{tag}.avro")
        self.io.write_bytes(lpath, avro.container_bytes(MANIFEST_FILE, [new] + manifests, metadata={
            "snapshot-id": str(sid), "parent-snapshot-id": str(parent["snapshot-id"]) if parent else "null",
            "sequence-number": str(seq), "format-version": str(FORMAT_VERSION)}))
        prev_total = int(parent["summary"].get("total-records", 0)) if parent else 0
        prev_files = int(parent["summary"].get("total-data-files", 0)) if parent else 0
        summary = {"operation": "append", "added-data-files": str(len(files)),
                   "added-records": str(new["added_rows_count"]),
                   "total-records": str(prev_total + new["added_rows_count"]),
                   "total-data-files": str(prev_files + len(files))}
        if commit_id is not None:
            summary[COMMIT_ID] = commit_id
        snap = {"snapshot-id": sid, "sequence-number": seq, "timestamp-ms": now, "manifest-list": lpath,
                "summary": summary, "schema-id": meta["current-schema-id"]}
        if parent is not None:
            snap["parent-snapshot-id"] = parent["snapshot-id"]
        meta["snapshots"].append(snap)
        meta["current-snapshot-id"] = sid
        meta["refs"] = {"main": {"snapshot-id": sid, "type": "branch"}}
        meta["last-sequence-number"] = seq
        meta["last-updated-ms"] = now
        meta["snapshot-log"].append({"timestamp-ms": now, "snapshot-id": sid})
        meta["metadata-log"].append({"timestamp-ms": self.meta["last-updated-ms"],
                                     "metadata-file": self._p("metadata", f"v{self.version}.metadata.json")})
        self._commit_metadata(meta)
        return snap

    def orphan_files(self) -> list[str]:
        """Data files under ``data/`` that no snapshot references (a writer died before its commit), as
        paths inside the table's filesystem."""
        inner = lambda p: self.io.resolve(p)[1]  # noqa: E731
        live = set()
        for s in self.snapshots():
            for m in self.manifests(s):
                for e in self.manifest_entries(m):
                    live.add(inner(e["data_file"]["file_path"]))
        return sorted(f for f in self.io.list(self._p("data"), recursive=True) if f not in live)


# ------------------------------------------------------------- sink and source
class IcebergSink:
    """Writes Arrow tables as Parquet data files of a table and commits them as append snapshots.

    The Parquet codec is the table's ``write.parquet.compression-codec`` property (Iceberg's table
    property for it), zstd when the table does not set one, as Iceberg's own writers default to."""

    CODEC_PROPERTY = "write.parquet.compression-codec"

    def __init__(self, table: IcebergTable, *, row_group_size: int = 64 * 1024):
        self.table = table
        self.row_group_size = row_group_size

    @property
    def codec(self) -> str:
        props = (self.table.meta or {}).get("properties", {})
        return str(props.get(self.CODEC_PROPERTY, "zstd")).lower()

    def write_files(self, tables: Iterable[pa.Table]) -> list[DataFile]:
        out = []
        target = _with_field_ids(self.table.arrow_schema(), self.table.schema())
        for t in tables:
            if t.num_rows == 0:
                continue
            t = t.select(target.names).cast(target)
            path = self.table._p("data", f"{uuid.uuid4().hex}.parquet")
            fs, inner, _ = self.table.io.resolve(path)
            if self.table._local:
                Path(inner).parent.mkdir(parents=True, exist_ok=True)
            with fs.open_output_stream(inner) as f:
                pq.write_table(t, f, row_group_size=self.row_group_size,
                               compression=None if self.codec == "uncompressed" else self.codec)
            size = fs.get_file_info(inner).size
            out.append(DataFile(path, t.num_rows, int(size)))
        return out

    def append(self, tables: Iterable[pa.Table], *, commit_id: str | None = None) -> dict | None:
        if commit_id is not None:
            done = self.table.refresh().find_commit(commit_id)
            if done is not None:
                return done
        files = self.write_files(tables)
        return self.table.append(files, commit_id=commit_id) if files else None


class IcebergSourceFactory:
    """Work items (row-group ranges) of a snapshot's data files, or of the appends after a cursor.

    ``mode="pinned"``: the files of ``snapshot_id`` (default: the current snapshot at construction).
    ``mode="continuous"``: the files appended after ``after_snapshot_id`` up to the snapshot current
    at construction; ``cursor`` is that end snapshot, the ``after_snapshot_id`` of the next scan."""

    def __init__(self, table: IcebergTable | str, *, mode: str = "pinned", snapshot_id: int | None = None,
                 after_snapshot_id: int | None = None, columns: Sequence[str] | None = None,
                 rows_per_item: int | None = None, max_concurrency: int = 4, cache=None):
        """``cache``: a ``data.file_cache.LocalFileCache`` through which data files on an object store are
        read (each downloaded once per node, identified by its path and size); local files are read in
        place."""
        self.table = table if isinstance(table, IcebergTable) else IcebergTable.load(table)
        self.cache = cache
        if mode not in ("pinned", "continuous"):
            raise ValueError("mode must be 'pinned' or 'continuous'")
        self.mode = mode
        cur = self.table.current_snapshot()
        self.cursor = cur["snapshot-id"] if cur else None
        if mode == "pinned":
            self.snapshot_id = snapshot_id if snapshot_id is not None else self.cursor
            self.files = self.table.plan_files(self.snapshot_id) if self.snapshot_id is not None else []
        else:
            self.snapshot_id = self.cursor
            self.files = self.table.appended_files(after_snapshot_id, self.cursor) if self.cursor is not None else []
        local = [self._local_path(f) for f in self.files]
        self._parquet = ParquetSourceFactory(local, columns=columns, rows_per_item=rows_per_item,
                                             max_concurrency=max_concurrency) if local else None

    def _local_path(self, f: DataFile) -> str:
        fs, inner, scheme = self.table.io.resolve(f.path)
        if scheme == "file":
            return inner
        if self.cache is None:
            raise ValueError("reading Iceberg data files from an object store needs a local cache "
                             f"(cache=LocalFileCache(...)); got {f.path}")
        return self.cache.local_path(f.path, f"size={f.file_size_in_bytes}")

    def plan(self) -> list[WorkItem]:
        return self._parquet.plan() if self._parquet else []

    def create_session(self) -> RecordRangeReadSession:
        if self._parquet is None:
            raise ValueError("the scan has no data files")
        return self._parquet.create_session()


__all__ = ["CommitConflict", "DataFile", "IcebergSink", "IcebergSourceFactory", "IcebergTable", "MANIFEST_ENTRY",
           "MANIFEST_FILE", "iceberg_schema"]
