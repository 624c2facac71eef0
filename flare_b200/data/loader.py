"""Background data loader with pinned host buffers and device prefetch.

A worker thread pulls assembled batches from a source, converts them with a
user transform into ``SparseBatch`` objects in pinned host memory and queues
them (bounded depth).  With ``device`` set, a second stage copies each batch to
the device on a dedicated CUDA stream ahead of use (the device-transfer stage
that the reference's dataloader leaves as a stub,
src/flare/data/pipeline/consumption/dataloader/device.py:8).  Iteration yields
batches that are safe to consume on the current stream.  ``close()`` (or
leaving a ``with`` block) stops the worker when the consumer ends early, so
the thread does not stay blocked on a full queue holding the source open.
"""
from __future__ import annotations

import queue
import threading
from collections.abc import Callable, Iterable, Iterator

import torch

from .synthetic import SparseBatch

_END = object()


class PrefetchLoader:
    def __init__(self, batches: Iterable, transform: Callable[[object], SparseBatch] | None = None, *,
                 depth: int = 4, pin_memory: bool = True, device: torch.device | None = None):
        self._src = iter(batches)
        self._transform = transform or (lambda b: b)
        self._q: queue.Queue = queue.Queue(maxsize=max(1, depth))
        self._pin = pin_memory and torch.cuda.is_available()
        self._device = device
        self._stream = torch.cuda.Stream(device=device) if device is not None and device.type == "cuda" else None
        self._error: BaseException | None = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._work, daemon=True)
        self._thread.start()

    def _put(self, item) -> bool:
        """Queue ``item`` unless the loader is closed first (False then)."""
        while not self._stop.is_set():
            try:
                self._q.put(item, timeout=0.05)
                return True
            except queue.Full:
                continue
        return False

    def _work(self) -> None:
        try:
            for raw in self._src:
                if self._stop.is_set():
                    return
                b = self._transform(raw)
                if self._pin:
                    b = b.pin_memory()
                if not self._put(b):
                    return
        except BaseException as exc:  # noqa: BLE001 - surfaced on the consumer side
            self._error = exc
        finally:
            self._put(_END)

    def close(self, timeout: float = 5.0) -> None:
        """Stop the worker and drop the batches it queued."""
        self._stop.set()
        while True:
            try:
                self._q.get_nowait()
            except queue.Empty:
                break
        self._thread.join(timeout=timeout)

    def __enter__(self) -> "PrefetchLoader":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __iter__(self) -> Iterator[SparseBatch]:
        pending = None
        while True:
            item = self._q.get()
            if item is _END:
                if pending is not None:
                    yield self._finish(pending)
                if self._error is not None:
                    raise self._error
                return
            staged = self._start_copy(item)
            if pending is not None:
                yield self._finish(pending)
            pending = staged

    def _start_copy(self, b: SparseBatch):
        if self._stream is None:
            return (b, None)
        with torch.cuda.stream(self._stream):
            d = b.to(self._device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._stream)
        return (d, ev)

    @staticmethod
    def _finish(p):
        b, ev = p
        if ev is not None:
            torch.cuda.current_stream(b.values.device).wait_event(ev)
            for t in (b.dense, b.labels, b.offsets, b.values):
                t.record_stream(torch.cuda.current_stream(t.device))
        return b


__all__ = ["PrefetchLoader"]
