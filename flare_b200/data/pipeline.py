"""Offline feature-production pipeline: raw records -> encoded Parquet training data.

    python -m flare_b200.data.run --config pipeline.yaml

Stages (host CPU; the hot loops are the native parser and encoders of
``csrc/etl.cpp``):

1. read: record files (plain, gzip or zstd), one record per line (TAB columns; the
   feature column holds ``code\\x03value`` items separated by ``\\x02``), in
   chunks of ``rows_per_file`` lines;
2. parse: ``ArrowRowParser`` on the chunk's Arrow string column (fixed,
   list and category features, plus direct / metadata columns);
3. encode: per output column an encoder: ``hash`` (value mod buckets),
   ``fnv_list`` (FNV-1a of a list, mod buckets), ``cross`` (seeded FNV-1a of
   two features, mod buckets), ``bucketize`` (bounds), ``fixed_width``,
   ``log1p`` / ``identity`` for dense values, ``intersect`` (list overlap
   count), ``category`` (vocabulary index);
4. publish: Parquet part files (``label``, ``d<i>`` float32, ``s<i>``
   list<int32>: the layout the training loaders read) grouped in publication
   windows.  A window is written into a temporary directory and renamed into
   place, then recorded in the publication manifest (atomic JSON), so a
   reader never sees a half-published window.

With ``run(workers=N)`` the inputs are split into N groups balanced by size
(largest first onto the least-loaded group) and encoded in parallel worker
processes; the coordinator renames and records their windows in input
order, and every input's written row count is checked against its decoded
records.

Operational state: a lease file (exclusive create, owner + expiry) keeps two
publishers off the same output; the manifest is the resume state (inputs
already published are skipped); on start, temporary windows left by a
crashed run are removed (crash reconciliation).

Reference behaviour: src/flare/data/pipeline/production/pipeline.py:46
(DataPipeline), publish/runner.py:291-334 (manifest), publication/
session.py:25 (leases), builder/resume_state_manager.py:45, stages/parse.py:89
and stages/feature_transform_split.py:24 (parse / encode),
recipes/recsys/data/heap_stream.py:44-64 (worker planning, size-balanced
groups) and category_values.py (vocabulary files).  Iceberg commits
are replaced by the window manifest (no Iceberg client in this build).
"""
from __future__ import annotations

import gzip
import os
import shutil
import socket
import time
import uuid
from collections.abc import Iterator
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from ..io.artifacts import read_json, write_json
from . import etl

MANIFEST = "_publication.json"
LEASE = "_lease.json"
TMP_PREFIX = ".window-"


@dataclass(frozen=True)
class DenseSpec:
    code: int
    transform: str = "identity"        # identity | log1p | bucketize | fixed_width
    bounds: tuple[float, ...] = ()
    width: float = 1.0


@dataclass(frozen=True)
class SparseSpec:
    kind: str                          # hash | fnv_list | cross | category | intersect
    codes: tuple[int, ...]
    buckets: int = 0
    seed: int = 0
    vocab: dict = field(default_factory=dict)
    default: int = 0


@dataclass(frozen=True)
class PipelineConfig:
    inputs: tuple[str, ...]
    output: str
    feature_column: int = 2
    label_code: int = 0
    dense: tuple[DenseSpec, ...] = ()
    sparse: tuple[SparseSpec, ...] = ()
    rows_per_file: int = 65536
    files_per_window: int = 4
    lease_seconds: float = 3600.0
    iceberg_table: str | None = None   # also commit every input's windows to this Iceberg table


# ------------------------------------------------------------------ reading
def _input_files(paths) -> list[str]:
    out = []
    for p in paths:
        if os.path.isdir(p):
            out += sorted(os.path.join(p, f) for f in os.listdir(p) if not f.startswith("."))
        else:
            out.append(p)
    return out


def _open_text(path: str):
    """Text stream of a record file: plain, gzip (``.gz``) or zstd (``.zst`` / ``.zstd``, Arrow's codec)."""
    if path.endswith(".gz"):
        return gzip.open(path, "rt", encoding="utf-8", newline="\n")
    if path.endswith((".zst", ".zstd")):
        import io

        import pyarrow as pa

        raw = pa.CompressedInputStream(pa.OSFile(path, "rb"), "zstd")
        return io.TextIOWrapper(io.BufferedReader(raw), encoding="utf-8", newline="\n")
    return open(path, "rt", encoding="utf-8", newline="\n")


def read_chunks(path: str, rows: int) -> Iterator[list[str]]:
    with _open_text(path) as f:
        chunk = []
        for line in f:
            if line.strip("\n"):
                chunk.append(line.rstrip("\n"))
            if len(chunk) == rows:
                yield chunk
                chunk = []
        if chunk:
            yield chunk


# ------------------------------------------------------------------ parse + encode
class FeatureProcessor:
    """Parse a chunk of records and encode the configured output columns."""

    def __init__(self, cfg: PipelineConfig):
        self.cfg = cfg
        fixed = {cfg.label_code: (1, True)}
        lists, cats = {}, {}
        for d in cfg.dense:
            fixed[d.code] = (1, True)
        for s in cfg.sparse:
            for c in s.codes:
                if s.kind == "category":
                    cats[c] = (s.vocab, s.default)
                elif s.kind in ("fnv_list", "intersect"):
                    lists[c] = False
                elif c not in fixed:
                    fixed[c] = (1, False)
        self.parser = etl.ArrowRowParser(feature_column=cfg.feature_column, fixed=fixed, lists=lists,
                                         categories=cats)

    def encode(self, lines: list[str]):
        import pyarrow as pa

        parsed = self.parser.parse(pa.array(lines, type=pa.string()))
        n = len(lines)
        cols = {"label": pa.array(np.where(parsed["fixed"][self.cfg.label_code][:, 0] == etl.NULL, 0.0,
                                           parsed["fixed"][self.cfg.label_code][:, 0]).astype(np.float32))}
        for i, d in enumerate(self.cfg.dense):
            v = parsed["fixed"][d.code][:, 0].astype(np.float32)
            missing = v == np.float32(etl.NULL)
            if d.transform == "log1p":
                out = np.log1p(np.abs(np.where(missing, 0.0, v))).astype(np.float32)
            elif d.transform == "bucketize":
                out = etl.bucketize(v, np.asarray(d.bounds, np.float32)).astype(np.float32)
            elif d.transform == "fixed_width":
                out = etl.fixed_width(v, d.width).astype(np.float32)
            else:
                out = np.where(missing, 0.0, v).astype(np.float32)
            cols[f"d{i}"] = pa.array(out)
        for i, s in enumerate(self.cfg.sparse):
            lens = np.ones(n, dtype=np.int32)
            if s.kind == "hash":
                vals = etl.hash_bucket(parsed["fixed"][s.codes[0]][:, 0], s.buckets)
            elif s.kind == "category":
                vals = parsed["categories"][s.codes[0]].astype(np.int64)
            elif s.kind == "cross":
                a = parsed["fixed"][s.codes[0]][:, 0]
                b = parsed["fixed"][s.codes[1]][:, 0]
                pair = etl.pack_fids(a, 0) ^ (b.astype(np.int64) * np.int64(0x9E3779B1))
                vals = (etl.fnv1a_seeded(pair & np.int64((1 << 62) - 1), s.seed) % np.uint64(max(s.buckets, 1))
                        ).astype(np.int64)
                vals[(a == etl.NULL) | (b == etl.NULL)] = etl.NULL
            elif s.kind == "fnv_list":
                v, o = parsed["lists"][s.codes[0]]
                vals = etl.fnv1a_lists(v, o, s.buckets).astype(np.int64)
                vals[np.diff(o) == 0] = etl.NULL
            elif s.kind == "intersect":
                va, oa = parsed["lists"][s.codes[0]]
                vb, ob = parsed["lists"][s.codes[1]]
                vals = etl.intersect_lists(va, oa, vb, ob).astype(np.int64)
            else:
                raise ValueError(f"unknown sparse encoder {s.kind!r}")
            keep = vals != etl.NULL
            lens = keep.astype(np.int32)
            offs = np.zeros(n + 1, dtype=np.int32)
            np.cumsum(lens, out=offs[1:])
            cols[f"s{i}"] = pa.ListArray.from_arrays(pa.array(offs), pa.array(vals[keep].astype(np.int32)))
        return pa.table(cols)


# ------------------------------------------------------------------ encode workers
def encode_input(cfg: PipelineConfig, path: str, out: str, proc: FeatureProcessor | None = None) -> list[dict]:
    """Encode one input into temporary window directories under ``out`` (renamed on commit).

    Checks that every decoded record is in the written Parquet files.
    """
    import pyarrow.parquet as pq

    proc = proc or FeatureProcessor(cfg)
    windows, cur, decoded = [], None, 0
    for lines in read_chunks(path, cfg.rows_per_file):
        if cur is None:
            cur = {"tmp": f"{TMP_PREFIX}{uuid.uuid4().hex[:12]}", "parts": 0, "rows": 0}
            (Path(out) / cur["tmp"]).mkdir()
        table = proc.encode(lines)
        pq.write_table(table, Path(out) / cur["tmp"] / f"part-{cur['parts']:05d}.parquet")
        cur["parts"] += 1
        cur["rows"] += table.num_rows
        decoded += len(lines)
        if cur["parts"] == cfg.files_per_window:
            windows.append(cur)
            cur = None
    if cur is not None:
        windows.append(cur)
    if sum(w["rows"] for w in windows) != decoded:
        raise RuntimeError(f"{path}: written rows differ from decoded records")
    return windows


def code_digest() -> str:
    """SHA-256 of the encoding code (this module and the ETL wrappers): every worker must run the same."""
    import hashlib

    h = hashlib.sha256()
    for mod in (__file__, etl.__file__):
        h.update(Path(mod).read_bytes())
    return h.hexdigest()


def encode_group(cfg: PipelineConfig, paths: list[str], out: str) -> list[tuple[str, list[dict]]]:
    """Worker process: encode a group of inputs (one feature processor for all)."""
    proc = FeatureProcessor(cfg)
    return [(p, encode_input(cfg, p, out, proc)) for p in paths]


def encode_group_measured(cfg: PipelineConfig, paths: list[str], out: str) -> tuple[list, dict]:
    """``encode_group`` plus the worker's wall / CPU seconds, peak RSS, host and code digest."""
    import resource

    t0, c0 = time.perf_counter(), time.process_time()
    res = encode_group(cfg, paths, out)
    return res, {"wall_seconds": time.perf_counter() - t0, "cpu_seconds": time.process_time() - c0,
                 "max_rss_bytes": resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * 1024,
                 "node": socket.gethostname(), "code_sha256": code_digest()}


def plan_groups(paths: list[str], workers: int) -> list[list[str]]:
    """Inputs into at most ``workers`` groups balanced by size: the largest remaining input goes to the
    least-loaded group (a heap of group loads); inputs keep their order inside a group."""
    import heapq

    heap = [(0, g) for g in range(min(workers, len(paths)))]
    groups: list[list[int]] = [[] for _ in heap]
    for i in sorted(range(len(paths)), key=lambda i: (-os.path.getsize(paths[i]), i)):
        load, g = heapq.heappop(heap)
        groups[g].append(i)
        heapq.heappush(heap, (load + os.path.getsize(paths[i]), g))
    return [[paths[i] for i in sorted(g)] for g in groups if g]


def plan_workers(*, cpus: int, memory_bytes: int, cpus_per_worker: int, memory_per_worker: int,
                 requested: int | None = None) -> int:
    """Encode workers that fit: leave ~3.5 % of the CPUs (at least one) to the driver and reserve at
    most 90 % of the memory; a request above that raises."""
    import math

    if cpus_per_worker <= 0 or memory_per_worker <= 0:
        raise ValueError("worker CPU and memory reservations must be positive")
    cpu_slots = (cpus - max(1, math.ceil(cpus * 0.035))) // cpus_per_worker
    avail = min(cpu_slots, int(memory_bytes * 0.9) // memory_per_worker)
    if avail < 1:
        raise ValueError("no encode worker fits the machine")
    if requested is not None and requested > avail:
        raise ValueError(f"requested {requested} workers, at most {avail} fit")
    return requested or avail


def load_category_values(category_files: dict[str, str], category_dir: str | Path
                         ) -> tuple[dict[str, dict[str, int]], frozenset[str]]:
    """Feature -> {value: index} from vocabulary files (one value per line, index = line order);
    features declared "auto" get no fixed vocabulary.  Empty or duplicate vocabularies raise."""
    cache: dict[str, dict[str, int]] = {}
    values, auto = {}, set()
    for feature, fname in category_files.items():
        if fname == "auto":
            auto.add(feature)
            continue
        if fname not in cache:
            vals = [v.strip() for v in (Path(category_dir) / fname).read_text(encoding="utf-8").splitlines()
                    if v.strip()]
            if not vals:
                raise ValueError(f"category vocabulary {fname} is empty")
            m = {v: i for i, v in enumerate(vals)}
            if len(m) != len(vals):
                raise ValueError(f"category vocabulary {fname} has duplicate values")
            cache[fname] = m
        values[feature] = cache[fname]
    return values, frozenset(auto)


# ------------------------------------------------------------------ publication state
class Lease:
    """Exclusive publisher lease on an output directory (owner + expiry; a stale lease is taken over).

    Every decision (acquire, renew, release) reads and writes the lease file under an exclusive
    ``flock`` on ``_lease.lock`` in the output directory, so of several publishers that find the same
    stale lease exactly one takes it over."""

    def __init__(self, out: Path, seconds: float):
        self.path = out / LEASE
        self.owner = f"{socket.gethostname()}:{os.getpid()}:{uuid.uuid4().hex[:8]}"
        self.seconds = seconds

    def _locked(self, fn):
        import fcntl

        with open(self.path.with_name(LEASE + ".lock"), "a+b") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                return fn(read_json(self.path) if self.path.exists() else None)
            finally:
                fcntl.flock(lock, fcntl.LOCK_UN)

    def acquire(self) -> None:
        def take(cur):
            if cur is not None and cur.get("owner") != self.owner and cur.get("expires", 0) > time.time():
                raise RuntimeError(f"output is leased by {cur.get('owner')} until {cur.get('expires')}")
            write_json(self.path, {"owner": self.owner, "expires": time.time() + self.seconds})
        self._locked(take)

    def renew(self) -> None:
        """Extend the expiry of a lease this publisher still owns (called at every commit)."""
        def extend(cur):
            if cur is None or cur.get("owner") != self.owner:
                raise RuntimeError(f"the lease on {self.path.parent} was taken over by "
                                   f"{cur.get('owner') if cur else 'nobody (released)'}")
            write_json(self.path, {"owner": self.owner, "expires": time.time() + self.seconds})
        self._locked(extend)

    def release(self) -> None:
        def drop(cur):
            if cur is not None and cur.get("owner") == self.owner:
                self.path.unlink(missing_ok=True)
        self._locked(drop)


class DataPipeline:
    def __init__(self, cfg: PipelineConfig, *, lineage=None):
        """``lineage``: an optional ``data.lineage.LineageRecorder``; every committed input is recorded
        as read (``file``), every published window (``parquet``, version = window directory, publication
        id = window id) and every Iceberg append (``iceberg``, version = snapshot id, publication id =
        the input's commit id) as published, and the recorder is flushed at the end of ``run``."""
        self.cfg = cfg
        self.out = Path(cfg.output)
        self.proc = FeatureProcessor(cfg)
        self.lineage = lineage

    def manifest(self) -> dict:
        p = self.out / MANIFEST
        return read_json(p) if p.exists() else {"windows": [], "inputs_done": []}

    def reconcile(self) -> list[str]:
        """Remove temporary windows of a crashed run; returns their names.  With an Iceberg table, every
        input already published gets its snapshot if the crash came between the two commits."""
        gone = []
        for d in self.out.glob(TMP_PREFIX + "*"):
            shutil.rmtree(d, ignore_errors=True)
            gone.append(d.name)
        if self.cfg.iceberg_table:
            man = self.manifest()
            for path in man["inputs_done"]:
                self._commit_iceberg(man, path)
        return gone

    def _iceberg(self):
        from .iceberg import IcebergTable

        if getattr(self, "_ice", None) is None:
            import pyarrow.parquet as pq

            files = self.published_files()
            if not files:
                return None
            schema = pq.read_schema(files[0])
            self._ice = IcebergTable.create(self.cfg.iceberg_table, schema, exist_ok=True)
        return self._ice

    def _commit_iceberg(self, man: dict, path: str) -> None:
        """One append snapshot per input, idempotent by the input's commit id."""
        import hashlib

        from .iceberg import DataFile

        table = self._iceberg()
        if table is None:
            return
        commit_id = "input:" + hashlib.sha256(path.encode()).hexdigest()[:32]
        if table.refresh().find_commit(commit_id) is not None:
            return
        files = []
        import pyarrow.parquet as pq

        for w in man["windows"]:
            if w["input"] != path:
                continue
            for i in range(w["parts"]):
                f = self.out / w["dir"] / f"part-{i:05d}.parquet"
                files.append(DataFile(str(f.absolute()), pq.ParquetFile(f).metadata.num_rows, f.stat().st_size))
        if files:
            snap = table.append(files, commit_id=commit_id)
            if self.lineage is not None:
                from .lineage import AssetRef

                self.lineage.output_published([AssetRef("iceberg", table.location, str(snap["snapshot-id"]))],
                                              commit_id)

    def run(self, workers: int = 1, *, audit_path: str | Path | None = None) -> dict:
        """Publish every input not yet in the manifest; ``workers > 1`` encodes in parallel processes.

        With ``audit_path`` the parallel run writes an audit JSON: rows per input, the code digest (every
        worker must report the same), worker nodes, summed wall / CPU seconds, peak worker RSS, groups
        and part files (the reference's heap-stream audit, recipes/recsys/data/heap_stream.py:207-226)."""
        self.out.mkdir(parents=True, exist_ok=True)
        lease = Lease(self.out, self.cfg.lease_seconds)
        lease.acquire()
        self._lease = lease
        try:
            self._check_catalog()
            self.reconcile()
            man = self.manifest()
            done = set(man["inputs_done"])
            todo = [f for f in _input_files(self.cfg.inputs) if f not in done]
            if workers <= 1 or len(todo) <= 1:
                for path in todo:
                    self._commit(man, path, encode_input(self.cfg, path, str(self.out)))
                return self._finished(man)
            import concurrent.futures as cf
            import multiprocessing as mp

            groups = plan_groups(todo, workers)
            t0 = time.perf_counter()
            expected, metrics, rows = code_digest(), [], {}
            with cf.ProcessPoolExecutor(max_workers=len(groups), mp_context=mp.get_context("spawn")) as ex:
                futs = [ex.submit(encode_group_measured, self.cfg, g, str(self.out)) for g in groups]
                for fut in futs:  # commit in group order; each group's inputs in order
                    res, m = fut.result()
                    if m["code_sha256"] != expected:
                        raise RuntimeError("encoding code differs across workers")
                    metrics.append(m)
                    for path, windows in res:
                        if path in rows:
                            raise RuntimeError(f"input {path} encoded by two groups")
                        rows[path] = sum(w["rows"] for w in windows)
                        self._commit(man, path, windows)
            if set(rows) != set(todo):
                raise RuntimeError("group coverage is incomplete")
            if audit_path is not None:
                write_json(audit_path, {
                    "source_rows": rows, "execution_engine": "process_groups", "code_sha256": expected,
                    "worker_nodes": sorted({m["node"] for m in metrics}), "total_rows": sum(rows.values()),
                    "groups": len(groups), "worker_seconds": sum(m["wall_seconds"] for m in metrics),
                    "worker_cpu_seconds": sum(m["cpu_seconds"] for m in metrics),
                    "max_worker_rss_bytes": max(m["max_rss_bytes"] for m in metrics),
                    "elapsed_before_commit": time.perf_counter() - t0,
                    "data_files": sum(w["parts"] for w in man["windows"] if w["input"] in rows)})
            return self._finished(man)
        finally:
            lease.release()

    def _check_catalog(self) -> None:
        """Publish the output's feature catalog, or check that an existing one has this config's digest."""
        from .feature_catalog import MANIFEST_NAME, FeatureCatalog, catalog_for

        cat = catalog_for(self.cfg)
        if (self.out / MANIFEST_NAME).exists():
            have = FeatureCatalog.from_manifest_dir(self.out)
            if have.config_digest != cat.config_digest:
                raise ValueError(f"{self.out} holds features of another configuration (digest "
                                 f"{have.config_digest[:12]}, this one {cat.config_digest[:12]})")
        else:
            cat.write_manifest(self.out)

    def _finished(self, man: dict) -> dict:
        if self.lineage is not None:
            self.lineage.flush()  # a failed export keeps the facts in the recorder and raises
        return man

    def _commit(self, man: dict, path: str, windows: list[dict]) -> None:
        """Rename an input's encoded windows into place and record them (the input is done)."""
        lease = getattr(self, "_lease", None)
        if lease is not None:
            lease.renew()  # a long run keeps its lease; a publisher that lost it stops before publishing
        for w in windows:
            wid = len(man["windows"])
            final = self.out / f"window-{wid:06d}"
            os.replace(self.out / w["tmp"], final)
            man["windows"].append({"id": wid, "dir": final.name, "parts": w["parts"], "rows": w["rows"],
                                   "input": path})
            write_json(self.out / MANIFEST, man)
            if self.lineage is not None:
                from .lineage import AssetRef

                self.lineage.output_published([AssetRef("parquet", str(self.out.absolute()), final.name)],
                                              f"window-{wid}")
        man["inputs_done"].append(path)
        write_json(self.out / MANIFEST, man)
        if self.lineage is not None:
            from .lineage import AssetRef

            self.lineage.inputs_read([AssetRef("file", str(Path(path).absolute()))])
        if self.cfg.iceberg_table:
            self._commit_iceberg(man, path)

    def published_files(self) -> list[str]:
        man = self.manifest()
        return [str(self.out / w["dir"] / f"part-{i:05d}.parquet") for w in man["windows"] for i in range(w["parts"])]


__all__ = ["DataPipeline", "DenseSpec", "FeatureProcessor", "Lease", "PipelineConfig", "SparseSpec", "code_digest",
           "encode_group", "encode_group_measured", "encode_input", "load_category_values", "plan_groups", "plan_workers", "read_chunks"]
