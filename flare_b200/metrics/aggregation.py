"""Windowed training metrics aggregated on the device, plus sinks.

``TrainMetricsWindow`` keeps the sampled predictions and labels of a window
(default 100 steps, reference: recipes/recsys/ranking/metrics/
train_metrics.py:127-326) in device buffers, and at the end of the window
computes exact AUC / GAUC (on the GPU when the data is there), calibration,
mean loss and throughput (valid samples / window wall time, reference:
src/flare/training/components/metrics/aggregation/sliding_window.py:8-23).
Metric names follow ``train/<metric>_<target>`` (reference:
recipes/recsys/ranking/metrics/sink.py:7-29).
"""
from __future__ import annotations

import collections
import json
import math
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Protocol

import torch

from .ranking import auc, calibration, gauc


@dataclass
class MetricWindow:
    start_time: float = field(default_factory=time.perf_counter)
    trained_sample_count: int = 0
    steps: int = 0

    def add(self, samples: int) -> None:
        self.trained_sample_count += int(samples)
        self.steps += 1

    def elapsed(self) -> float:
        return time.perf_counter() - self.start_time

    def throughput_samples(self) -> float:
        dt = self.elapsed()
        return self.trained_sample_count / dt if dt > 0 else 0.0


class MetricSink(Protocol):
    def write(self, step: int, metrics: dict[str, float]) -> None: ...


class ConsoleSink:
    def __init__(self, prefix: str = "[TrainMetrics]"):
        self.prefix = prefix

    def write(self, step: int, metrics: dict[str, float]) -> None:
        body = " ".join(f"{k}={v:.6g}" for k, v in sorted(metrics.items()))
        print(f"{self.prefix} step={step} {body}", flush=True)


class JsonlSink:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)

    def write(self, step: int, metrics: dict[str, float]) -> None:
        with self.path.open("a") as f:
            f.write(json.dumps({"step": step, **metrics}) + "\n")


class TensorBoardSink:
    """Writes scalars with tensorboardX or torch.utils.tensorboard when installed."""

    def __init__(self, logdir: str | Path):
        try:
            from tensorboardX import SummaryWriter  # type: ignore
        except ImportError:
            try:
                from torch.utils.tensorboard import SummaryWriter  # type: ignore
            except ImportError as exc:  # pragma: no cover - depends on the image
                raise RuntimeError("no TensorBoard writer installed; use JsonlSink") from exc
        self.writer = SummaryWriter(str(logdir))

    def write(self, step: int, metrics: dict[str, float]) -> None:
        for k, v in metrics.items():
            self.writer.add_scalar(k, v, step)
        self.writer.flush()


class TrainMetricsWindow:
    def __init__(self, targets: tuple[str, ...] = ("ctr",), window_steps: int = 100, capacity: int = 1 << 22,
                 device: torch.device | None = None, sinks: list | None = None, negative_factor: float = 0.0,
                 distributed: bool | None = None, group=None, background: bool = False, max_pending: int = 2,
                 merge: str = "allgather"):
        """``distributed``: merge every rank's window into one exact AUC / GAUC / calibration / loss /
        throughput (default: when a process group of more than one rank is up).  Every rank must then
        call ``update`` for the same steps, since the flush is a collective.  ``merge`` picks how the
        ranks' windows are merged (``metrics.distributed.distributed_metrics``: ``"allgather"``, or
        ``"partitioned"`` for windows too large to hold on every rank).

        ``background`` (rank-local windows): a finished window is copied on the device and its metrics
        are computed by one worker thread while training goes on; at most ``max_pending`` windows wait
        (the next flush blocks on the oldest, so a slow metric slows training instead of queueing
        without bound).  Results reach the sinks in window order and ``completed``; ``drain()`` waits
        for all of them.  Reference behaviour: bounded background pending windows of the train
        metrics aggregator (recipes/recsys/ranking/metrics/train_metrics.py:127-326)."""
        self.targets = targets
        if merge not in ("allgather", "partitioned"):
            raise ValueError(f"merge must be 'allgather' or 'partitioned', got {merge!r}")
        self.group = group
        self.distributed = distributed
        self.merge = merge
        self.window_steps = window_steps
        self.device = device or torch.device("cpu")
        T = len(targets)
        self.scores = torch.empty(capacity, T, dtype=torch.float32, device=self.device)
        self.labels = torch.empty(capacity, T, dtype=torch.float32, device=self.device)
        self.groups = torch.empty(capacity, dtype=torch.int64, device=self.device)
        self.loss_sum = torch.zeros((), dtype=torch.float64, device=self.device)
        self.n = 0
        self.has_groups = False
        self.window = MetricWindow()
        self.sinks = sinks or []
        self.negative_factor = negative_factor
        self.total_steps = 0
        self.background, self.max_pending = bool(background), max(1, int(max_pending))
        self._pool = None
        self._pending: collections.deque = collections.deque()
        self.completed: list[dict] = []

    def update(self, logits: torch.Tensor, labels: torch.Tensor, *, loss_sum: torch.Tensor | float | None = None,
               groups: torch.Tensor | None = None, valid_count: int | None = None) -> dict | None:
        B = logits.shape[0] if valid_count is None else valid_count
        k = min(B, self.scores.shape[0] - self.n)
        if k > 0:
            self.scores[self.n:self.n + k] = torch.sigmoid(logits[:k].float()).reshape(k, -1)
            self.labels[self.n:self.n + k] = labels[:k].float().reshape(k, -1)
            if groups is not None:
                self.groups[self.n:self.n + k] = groups[:k].to(torch.int64)
                self.has_groups = True
            self.n += k
        if loss_sum is not None:
            self.loss_sum += loss_sum if not torch.is_tensor(loss_sum) else loss_sum.to(self.loss_sum.device).double().reshape(())
        self.window.add(B)
        self.total_steps += 1
        if self.window.steps >= self.window_steps:
            return self.flush()
        return None

    def _is_distributed(self) -> bool:
        if self.distributed is not None:
            return self.distributed
        import torch.distributed as dist

        return dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1

    def flush(self) -> dict | None:
        """End the window: its metrics (None when a background worker computes them)."""
        out: dict[str, float] = {}
        n = self.n
        if self._is_distributed():
            from .distributed import _max_scalar, _sum_scalars, distributed_metrics

            grouped = self.has_groups
            for t, name in enumerate(self.targets):
                m = distributed_metrics(self.scores[:n, t], self.labels[:n, t], self.groups[:n] if grouped else None,
                                        negative_factor=self.negative_factor, group=self.group, merge=self.merge)
                for k, v in m.items():
                    out[f"train/{k}_{name}"] = v
            elapsed = self.window.elapsed()
            # loss and samples summed over the ranks, wall time of the slowest rank
            loss, samples = _sum_scalars([float(self.loss_sum), float(self.window.trained_sample_count)],
                                         self.group, self.loss_sum.device)
            slowest = _max_scalar(elapsed, self.group, self.loss_sum.device)
            out["train/loss"] = loss / max(samples, 1.0)
            out["train/throughput_samples"] = samples / max(slowest, 1e-9)
        elif self.background:
            snap = (self.scores[:n].clone(), self.labels[:n].clone(),
                    self.groups[:n].clone() if self.has_groups else None, self.loss_sum.clone(),
                    self.window.trained_sample_count, self.window.throughput_samples(), self.total_steps)
            ev = None
            if self.device.type == "cuda":
                ev = torch.cuda.Event()
                ev.record()
            while len(self._pending) >= self.max_pending:
                self._pending.popleft().result()
            if self._pool is None:
                from concurrent.futures import ThreadPoolExecutor

                self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="metrics-window")
            self._pending.append(self._pool.submit(self._background_window, snap, ev))
            self._reset()
            return None
        else:
            out = self._local_metrics(self.scores[:n], self.labels[:n], self.groups[:n] if self.has_groups else None,
                                      float(self.loss_sum), self.window.trained_sample_count,
                                      self.window.throughput_samples())
        self._emit(self.total_steps, out)
        self._reset()
        return out

    def _local_metrics(self, scores, labels, groups, loss_sum: float, samples: int, throughput: float) -> dict:
        out: dict[str, float] = {}
        if scores.shape[0]:
            for t, name in enumerate(self.targets):
                s, y = scores[:, t], labels[:, t]
                out[f"train/auc_{name}"] = auc(s, y)
                out[f"train/calibration_{name}"] = calibration(s, y)
                if groups is not None:
                    out[f"train/gauc_{name}"] = gauc(s, y, groups, self.negative_factor)
        out["train/loss"] = loss_sum / max(samples, 1)
        out["train/throughput_samples"] = throughput
        return out

    def _background_window(self, snap, ev) -> dict:
        scores, labels, groups, loss, samples, throughput, step = snap
        if ev is not None:
            ev.synchronize()  # the copies were queued on the training stream
        out = self._local_metrics(scores, labels, groups, float(loss), samples, throughput)
        self._emit(step, out)
        self.completed.append(out)
        return out

    def _emit(self, step: int, out: dict) -> None:
        for sink in self.sinks:
            sink.write(step, {k: v for k, v in out.items() if not (isinstance(v, float) and math.isnan(v))})

    def _reset(self) -> None:
        self.n = 0
        self.has_groups = False
        self.loss_sum.zero_()
        self.window = MetricWindow()

    def drain(self) -> list[dict]:
        """Wait for every background window; returns all completed window results (in order)."""
        while self._pending:
            self._pending.popleft().result()
        return list(self.completed)

    def close(self) -> None:
        self.drain()
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None


__all__ = ["ConsoleSink", "JsonlSink", "MetricSink", "MetricWindow", "TensorBoardSink", "TrainMetricsWindow"]
