"""Diagnostics: asynchronous JSONL execution trace, state fingerprints, timers.

* ``JsonlExecutionTracer`` writes semantic events (one JSON object per line,
  one file per stage) from a background thread through a bounded queue, so the
  training loop never blocks on file I/O; events carry a monotonic sequence
  number; tensors in an event are summarised (shape, dtype, finite / NaN / Inf
  counts, min / max / mean) instead of dumped.  Reference:
  src/flare/runtime/diagnostics/execution_trace.py:34-182.
* ``fingerprint_state`` hashes every tensor (name, shape, dtype, bytes) with
  BLAKE2b, giving a per-leaf and a combined digest (reference:
  src/flare/runtime/diagnostics/state_audit.py:11).
* ``StepTimer`` times device work with CUDA events (max over ranks when
  distributed); ``median_duration_seconds`` for host timings.
"""
from __future__ import annotations

import hashlib
import json
import queue
import statistics
import threading
import time
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch


def summarize_tensor(t: torch.Tensor) -> dict:
    x = t.detach()
    out = {"shape": list(x.shape), "dtype": str(x.dtype).replace("torch.", "")}
    if x.is_floating_point() and x.numel():
        xf = x.float()
        fin = torch.isfinite(xf)
        out.update(finite=int(fin.sum()), nan=int(torch.isnan(xf).sum()), inf=int(torch.isinf(xf).sum()))
        if bool(fin.any()):
            v = xf[fin]
            out.update(min=float(v.min()), max=float(v.max()), mean=float(v.mean()))
    elif x.numel():
        out.update(min=int(x.min()), max=int(x.max()))
    return out


def _jsonable(v: Any):
    if isinstance(v, torch.Tensor):
        return summarize_tensor(v)
    if isinstance(v, Mapping):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, (int, float, str, bool)) or v is None:
        return v
    return repr(v)


class JsonlExecutionTracer:
    def __init__(self, directory: str | Path, *, rank: int = 0, max_queue: int = 10000, enabled: bool = True):
        self.enabled = enabled
        self.dir = Path(directory)
        self.rank = rank
        self._seq = 0
        self._q: queue.Queue = queue.Queue(maxsize=max_queue)
        self.dropped = 0
        self._files: dict[str, Any] = {}
        self._thread = None
        if enabled:
            self.dir.mkdir(parents=True, exist_ok=True)
            self._thread = threading.Thread(target=self._drain, daemon=True)
            self._thread.start()

    def emit(self, stage: str, event: str, **fields) -> None:
        """Record one event; never blocks (drops and counts when the queue is full)."""
        if not self.enabled:
            return
        self._seq += 1
        rec = {"seq": self._seq, "time": time.time(), "rank": self.rank, "stage": stage, "event": event,
               **_jsonable(fields)}
        try:
            self._q.put_nowait(rec)
        except queue.Full:
            self.dropped += 1

    def _drain(self) -> None:
        while True:
            rec = self._q.get()
            if rec is None:
                break
            f = self._files.get(rec["stage"])
            if f is None:
                f = (self.dir / f"{rec['stage']}.rank{self.rank}.jsonl").open("a")
                self._files[rec["stage"]] = f
            f.write(json.dumps(rec) + "\n")
            if self._q.empty():
                f.flush()

    def close(self) -> None:
        if self._thread is not None:
            self._q.put(None)
            self._thread.join(timeout=10)
            self._thread = None
        for f in self._files.values():
            f.close()
        self._files.clear()


def fingerprint_state(state: Mapping[str, torch.Tensor]) -> dict:
    leaves = {}
    combined = hashlib.blake2b(digest_size=32)
    for name in sorted(state):
        t = state[name].detach().contiguous().cpu()
        h = hashlib.blake2b(digest_size=32)
        h.update(f"{name}|{tuple(t.shape)}|{t.dtype}|".encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
        leaves[name] = h.hexdigest()
        combined.update(leaves[name].encode())
    return {"leaves": leaves, "digest": combined.hexdigest(), "count": len(leaves)}


def median_duration_seconds(durations) -> float:
    d = [float(x) for x in durations]
    if not d:
        raise ValueError("no durations")
    return statistics.median(d)


class StepTimer:
    """CUDA-event timing of a region on the current stream; ``stop`` returns ms."""

    def __init__(self, device: torch.device | None = None):
        self.device = device
        self._start = torch.cuda.Event(enable_timing=True)
        self._stop = torch.cuda.Event(enable_timing=True)

    def start(self) -> None:
        self._start.record()

    def stop(self, max_over_ranks: bool = True) -> float:
        self._stop.record()
        self._stop.synchronize()
        ms = self._start.elapsed_time(self._stop)
        if max_over_ranks:
            from ..parallel.dist import max_over_ranks as _max

            ms = _max(ms)
        return ms


__all__ = ["JsonlExecutionTracer", "StepTimer", "fingerprint_state", "median_duration_seconds", "summarize_tensor"]
