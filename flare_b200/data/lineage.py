"""Data lineage: asset-level facts of a run (inputs read, outputs published), exported in batches.

Facts name assets, never data: ``InputRead(asset)`` and ``OutputPublished(asset, publication_id)``
with ``AssetRef(namespace, name, version)`` (a file, a table at a snapshot, a published window).
``LineageRecorder`` collects them for one run (``LineageContext(run_id, operation_id)``):

* a fact already pending, or exported within the last ``coalesce_window`` distinct facts, is dropped
  (a fixed input snapshot read on every batch is one fact), and a repeated fact refreshes its place
  in that window;
* at most ``max_pending_events`` facts wait; recording one more exports the pending ones first;
* ``flush()`` exports the pending facts in the order they were first recorded, through the exporter
  the factory creates on the first export (a recorder that records nothing never creates one); a
  failed export keeps the facts pending and raises, so a later flush retries them;
* ``close()`` (once; later calls do nothing) flushes, closes the exporter and raises an
  ``ExceptionGroup`` of every failure; afterwards recording is an error.

Recording and flushing are serialised by a lock, so threads of one process share a recorder.
``JsonlLineageExporter`` appends each export as JSON lines to a file.  The feature pipeline records
its inputs and its published windows / Iceberg snapshots when given a recorder
(``data.pipeline.DataPipeline(cfg, lineage=...)``).

Reference behaviour: src/flare/data/contracts/lineage.py (facts, context, exporter protocols) and
src/flare/data/pipeline/lineage.py (bounded, coalescing recorder with explicit delivery), written
here for a synchronous pipeline.
"""
from __future__ import annotations

import json
import threading
from collections import OrderedDict
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Protocol, runtime_checkable


def _canonical(value, what: str) -> None:
    if not isinstance(value, str) or not value or value.strip() != value:
        raise ValueError(f"{what} must be a non-empty string without surrounding blanks")


@dataclass(frozen=True)
class AssetRef:
    namespace: str
    name: str
    version: str | None = None

    def __post_init__(self) -> None:
        _canonical(self.namespace, "asset namespace")
        _canonical(self.name, "asset name")
        if self.version is not None:
            _canonical(self.version, "asset version")

    def to_dict(self) -> dict:
        return {"namespace": self.namespace, "name": self.name, "version": self.version}


@dataclass(frozen=True)
class LineageContext:
    run_id: str
    operation_id: str

    def __post_init__(self) -> None:
        _canonical(self.run_id, "lineage run id")
        _canonical(self.operation_id, "lineage operation id")


@dataclass(frozen=True)
class InputRead:
    asset: AssetRef

    def __post_init__(self) -> None:
        if not isinstance(self.asset, AssetRef):
            raise TypeError("a lineage input names an AssetRef")


@dataclass(frozen=True)
class OutputPublished:
    asset: AssetRef
    publication_id: str

    def __post_init__(self) -> None:
        if not isinstance(self.asset, AssetRef):
            raise TypeError("a lineage output names an AssetRef")
        _canonical(self.publication_id, "publication id")


LineageEvent = InputRead | OutputPublished


@runtime_checkable
class LineageExporter(Protocol):
    def export(self, events: tuple[LineageEvent, ...]) -> None: ...

    def close(self) -> None: ...


def event_to_dict(event: LineageEvent, context: LineageContext | None = None) -> dict:
    d = {"kind": "input_read" if isinstance(event, InputRead) else "output_published", "asset": event.asset.to_dict()}
    if isinstance(event, OutputPublished):
        d["publication_id"] = event.publication_id
    if context is not None:
        d.update(run_id=context.run_id, operation_id=context.operation_id)
    return d


class JsonlLineageExporter:
    """Appends every exported fact as one JSON line (with the run's ids) to ``path``."""

    def __init__(self, path: str | Path, context: LineageContext):
        self.path, self.context = Path(path), context
        self.path.parent.mkdir(parents=True, exist_ok=True)

    def export(self, events: tuple[LineageEvent, ...]) -> None:
        with open(self.path, "a", encoding="utf-8") as f:
            for e in events:
                f.write(json.dumps(event_to_dict(e, self.context), sort_keys=True) + "\n")

    def close(self) -> None:
        pass


class LineageRecorder:
    def __init__(self, exporter_factory: Callable[[LineageContext], LineageExporter], context: LineageContext, *,
                 max_pending_events: int = 1024, coalesce_window: int = 4096):
        if not callable(exporter_factory):
            raise TypeError("exporter_factory must be callable with the lineage context")
        if not isinstance(context, LineageContext):
            raise TypeError("context must be a LineageContext")
        for v in (max_pending_events, coalesce_window):
            if type(v) is not int or v <= 0:
                raise ValueError("lineage limits must be positive integers")
        self._factory, self.context = exporter_factory, context
        self._capacity, self._window = max_pending_events, coalesce_window
        self._pending: OrderedDict[LineageEvent, None] = OrderedDict()
        self._seen: OrderedDict[LineageEvent, None] = OrderedDict()
        self._exporter: LineageExporter | None = None
        self._lock = threading.RLock()
        self._closed = False
        self._close_done = False

    @property
    def pending_events(self) -> tuple[LineageEvent, ...]:
        with self._lock:
            return tuple(self._pending)

    def _known(self, event: LineageEvent) -> bool:
        if event in self._seen:
            self._seen.move_to_end(event)
            return True
        return event in self._pending

    def _record(self, events: Sequence[LineageEvent]) -> None:
        with self._lock:
            if self._closed:
                raise RuntimeError("lineage recorder is closed")
            for e in events:
                if self._known(e):
                    continue
                while len(self._pending) >= self._capacity:
                    self._flush_locked()
                    if self._known(e):
                        break
                else:
                    self._pending[e] = None

    def inputs_read(self, assets: Sequence[AssetRef]) -> None:
        self._record([InputRead(a) for a in assets])

    def output_published(self, assets: Sequence[AssetRef], publication_id: str) -> None:
        self._record([OutputPublished(a, publication_id) for a in assets])

    def _flush_locked(self) -> None:
        batch = tuple(self._pending)
        if not batch:
            return
        if self._exporter is None:
            exporter = self._factory(self.context)
            if not isinstance(exporter, LineageExporter):
                raise TypeError("the lineage exporter factory must return an exporter (export, close)")
            self._exporter = exporter
        self._exporter.export(batch)  # on failure the facts stay pending
        for e in batch:
            del self._pending[e]
            self._seen[e] = None
            self._seen.move_to_end(e)
            if len(self._seen) > self._window:
                self._seen.popitem(last=False)

    def flush(self) -> None:
        with self._lock:
            if self._closed:
                raise RuntimeError("lineage recorder is closed")
            self._flush_locked()

    def close(self) -> None:
        with self._lock:
            if self._close_done:
                return
            self._closed = True
            self._close_done = True
            failures: list[Exception] = []
            try:
                self._flush_locked()
            except Exception as e:  # noqa: BLE001 - reported together below
                failures.append(e)
            if self._exporter is not None:
                try:
                    self._exporter.close()
                except Exception as e:  # noqa: BLE001
                    failures.append(e)
            if failures:
                raise ExceptionGroup("lineage close failed", failures)


__all__ = ["AssetRef", "InputRead", "JsonlLineageExporter", "LineageContext", "LineageEvent", "LineageExporter",
           "LineageRecorder", "OutputPublished", "event_to_dict"]
