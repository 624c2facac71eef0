"""Offline feature-production pipeline: raw records -> encoded Parquet training data.

    python -m flare_b200.data.run --config pipeline.yaml

Stages (host CPU; the hot loops are the native parser and encoders of
``csrc/etl.cpp``):

1. read: record files (plain or gzip), one record per line (TAB columns; the
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

Operational state: a lease file (exclusive create, owner + expiry) keeps two
publishers off the same output; the manifest is the resume state (inputs
already published are skipped); on start, temporary windows left by a
crashed run are removed (crash reconciliation).

Reference behaviour: src/flare/data/pipeline/production/pipeline.py:46
(DataPipeline), publish/runner.py:291-334 (manifest), publication/
session.py:25 (leases), builder/resume_state_manager.py:45, stages/parse.py:89
and stages/feature_transform_split.py:24 (parse / encode).  Iceberg commits
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


# ------------------------------------------------------------------ reading
def _input_files(paths) -> list[str]:
    out = []
    for p in paths:
        if os.path.isdir(p):
            out += sorted(os.path.join(p, f) for f in os.listdir(p) if not f.startswith("."))
        else:
            out.append(p)
    return out


def read_chunks(path: str, rows: int) -> Iterator[list[str]]:
    opener = gzip.open if path.endswith(".gz") else open
    with opener(path, "rt", encoding="utf-8", newline="\n") as f:
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


# ------------------------------------------------------------------ publication state
class Lease:
    """Exclusive publisher lease on an output directory (owner + expiry; a stale lease is taken over)."""

    def __init__(self, out: Path, seconds: float):
        self.path = out / LEASE
        self.owner = f"{socket.gethostname()}:{os.getpid()}:{uuid.uuid4().hex[:8]}"
        self.seconds = seconds

    def acquire(self) -> None:
        body = {"owner": self.owner, "expires": time.time() + self.seconds}
        try:
            write_json(self.path, body, exclusive=True)
            return
        except FileExistsError:
            cur = read_json(self.path)
            if cur.get("expires", 0) > time.time():
                raise RuntimeError(f"output is leased by {cur.get('owner')} until {cur.get('expires')}")
        write_json(self.path, body)  # expired: take over

    def release(self) -> None:
        try:
            if read_json(self.path).get("owner") == self.owner:
                self.path.unlink()
        except FileNotFoundError:
            pass


class DataPipeline:
    def __init__(self, cfg: PipelineConfig):
        self.cfg = cfg
        self.out = Path(cfg.output)
        self.proc = FeatureProcessor(cfg)

    def manifest(self) -> dict:
        p = self.out / MANIFEST
        return read_json(p) if p.exists() else {"windows": [], "inputs_done": []}

    def reconcile(self) -> list[str]:
        """Remove temporary windows of a crashed run; returns their names."""
        gone = []
        for d in self.out.glob(TMP_PREFIX + "*"):
            shutil.rmtree(d, ignore_errors=True)
            gone.append(d.name)
        return gone

    def run(self) -> dict:
        self.out.mkdir(parents=True, exist_ok=True)
        lease = Lease(self.out, self.cfg.lease_seconds)
        lease.acquire()
        try:
            self.reconcile()
            man = self.manifest()
            done = set(man["inputs_done"])
            todo = [f for f in _input_files(self.cfg.inputs) if f not in done]
            for path in todo:
                self._publish_input(path, man)
            return man
        finally:
            lease.release()

    def _publish_input(self, path: str, man: dict) -> None:
        import pyarrow.parquet as pq

        window, parts, rows = None, 0, 0
        wid = len(man["windows"])

        def commit():
            nonlocal window, parts, rows, wid
            final = self.out / f"window-{wid:06d}"
            os.replace(window, final)
            man["windows"].append({"id": wid, "dir": final.name, "parts": parts, "rows": rows, "input": path})
            write_json(self.out / MANIFEST, man)
            window, parts, rows, wid = None, 0, 0, wid + 1

        for lines in read_chunks(path, self.cfg.rows_per_file):
            if window is None:
                window = self.out / f"{TMP_PREFIX}{uuid.uuid4().hex[:12]}"
                window.mkdir()
            table = self.proc.encode(lines)
            pq.write_table(table, window / f"part-{parts:05d}.parquet")
            parts += 1
            rows += table.num_rows
            if parts == self.cfg.files_per_window:
                commit()
        if window is not None:
            commit()
        man["inputs_done"].append(path)
        write_json(self.out / MANIFEST, man)

    def published_files(self) -> list[str]:
        man = self.manifest()
        return [str(self.out / w["dir"] / f"part-{i:05d}.parquet") for w in man["windows"] for i in range(w["parts"])]


__all__ = ["DataPipeline", "DenseSpec", "FeatureProcessor", "Lease", "PipelineConfig", "SparseSpec", "read_chunks"]
