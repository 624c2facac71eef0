"""Input-pipeline throughput harness: reader lanes -> input ranks -> throughput sinks (CPU).

    python -m flare_b200.benchmarks.throughput --input-workers 2 --reader-workers 4 --steps 20

Measures how fast the host side of training (Parquet range reads, batch
assembly, Arrow -> keyed-jagged conversion, first-occurrence id dedup) can
feed ``samples_per_input_step`` samples to each input rank, without any GPU.
``reader_workers`` reader lanes (threads) read the planned work items
round-robin; each input rank interleaves ``reader_workers / input_workers``
lanes, assembles fixed-size batches (completion policy ``pad`` keeps every
step full-size), converts them and hands the valid-sample count to its
``ThroughputSink``, which records arrival times.  ``summarize_sink_reports``
turns the sink reports into end-to-end and arrival-window samples/s and the
p50/p95 step interval.

Reference behaviour: recipes/recsys/ranking/benchmark/runner.py:79 (graph),
throughput_sink.py:27 (sink), metrics.py:10-108 (summary keys).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import queue
import tempfile
import threading
import time
from collections.abc import Mapping, Sequence
from typing import Any

import numpy as np
import torch

from ..data.schema import TrainingFeatureLayout, table_to_training_dict
from ..data.sources import BatchAssembler, ParquetSourceFactory
from ..ops.sparse import unique_first_occurrence


class ThroughputSink:
    """Records the arrival time and valid-sample count of every step of one input rank."""

    def __init__(self, rank: int, world_size: int, max_steps: int | None = None):
        if max_steps is not None and max_steps <= 0:
            raise ValueError("max_steps must be positive")
        self.rank, self.world_size, self.max_steps = rank, world_size, max_steps
        self.arrivals: list[float] = []
        self.counts: list[int] = []

    @property
    def done(self) -> bool:
        return self.max_steps is not None and len(self.counts) >= self.max_steps

    def consume(self, valid_samples: int) -> None:
        if int(valid_samples) <= 0:
            raise ValueError("a throughput sink needs positive valid samples per step")
        self.arrivals.append(time.perf_counter())
        self.counts.append(int(valid_samples))

    def report(self) -> dict[str, Any]:
        gaps = [b - a for a, b in zip(self.arrivals[:-1], self.arrivals[1:])]
        return {"rank": self.rank, "world_size": self.world_size, "graph_steps": len(self.counts),
                "step_valid_samples": list(self.counts), "valid_samples": sum(self.counts),
                "step_intervals": gaps, "measured_duration_seconds": float(sum(gaps))}


def _positive_int(x) -> bool:
    return type(x) is int and x > 0


def summarize_sink_reports(reports: Sequence[Mapping[str, Any]], *, input_workers: int, reader_workers: int,
                           samples_per_input_step: int, global_batch_size: int, steps: int,
                           wall_seconds: float) -> dict[str, Any]:
    """Validate the sink reports against the requested topology and summarise throughput."""
    if not all(_positive_int(v) for v in (input_workers, reader_workers, samples_per_input_step,
                                          global_batch_size, steps)):
        raise ValueError("worker counts, samples per step, global batch and steps must be positive integers")
    if global_batch_size != samples_per_input_step * input_workers:
        raise ValueError("global_batch_size must equal samples_per_input_step x input_workers")
    if reader_workers % input_workers:
        raise ValueError("reader_workers must be a multiple of input_workers")
    if not (math.isfinite(wall_seconds) and wall_seconds > 0):
        raise ValueError("wall_seconds must be finite and positive")
    if sorted(r["rank"] for r in reports) != list(range(input_workers)):
        raise ValueError("sink reports must cover every input rank exactly once")
    gaps_all: list[float] = []
    total = window = 0
    durations = []
    for r in reports:
        if r["world_size"] != input_workers or r["graph_steps"] != steps:
            raise ValueError(f"sink {r['rank']}: topology or completed steps differ from the request")
        counts = r["step_valid_samples"]
        if len(counts) != steps or any(c != samples_per_input_step for c in counts):
            raise ValueError(f"sink {r['rank']}: every step must carry samples_per_input_step valid samples")
        if sum(counts) != r["valid_samples"]:
            raise ValueError(f"sink {r['rank']}: total disagrees with the per-step counts")
        gaps = r["step_intervals"]
        if len(gaps) != steps - 1 or any(not (math.isfinite(g) and g > 0) for g in gaps):
            raise ValueError(f"sink {r['rank']}: arrival intervals are invalid or incomplete")
        if not math.isclose(r["measured_duration_seconds"], sum(gaps), rel_tol=1e-6, abs_tol=1e-6):
            raise ValueError(f"sink {r['rank']}: duration disagrees with the arrival intervals")
        durations.append(r["measured_duration_seconds"])
        gaps_all += gaps
        total += sum(counts)
        window += sum(counts[1:])
    e2e = total / wall_seconds
    win_s = max(durations)
    win_rate = window / win_s if steps > 1 and win_s > 0 else None
    return {
        "reader_workers": reader_workers, "input_workers": input_workers, "sink_workers": input_workers,
        "samples_per_input_step": samples_per_input_step, "global_batch_size": global_batch_size,
        "reader_interleave_factor": reader_workers // input_workers, "graph_steps": steps,
        "valid_samples": total, "wall_seconds": wall_seconds,
        "end_to_end_aggregate_samples_per_second": e2e,
        "end_to_end_per_input_samples_per_second": e2e / input_workers,
        "arrival_window_samples": window, "arrival_window_seconds": win_s,
        "arrival_window_aggregate_samples_per_second": win_rate,
        "arrival_window_per_input_samples_per_second": None if win_rate is None else win_rate / input_workers,
        "p50_step_seconds": float(np.percentile(gaps_all, 50)) if gaps_all else None,
        "p95_step_seconds": float(np.percentile(gaps_all, 95)) if gaps_all else None,
    }


# ----------------------------------------------------------------- synthetic files
def write_synthetic_parquet(directory: str, *, files: int = 4, rows_per_file: int = 65536, num_sparse: int = 26,
                            num_dense: int = 13, max_bag: int = 16, vocab: int = 1_000_000, row_group: int = 8192,
                            seed: int = 0) -> list[str]:
    """DLRM-shaped Parquet files: ``label``, ``d0..`` float32, ``s0..`` list<int32> (Zipf ids)."""
    import pyarrow as pa
    import pyarrow.parquet as pq

    from ..data.synthetic import zipf_ids

    g = torch.Generator().manual_seed(seed)
    paths = []
    for k in range(files):
        cols = {"label": pa.array((torch.rand(rows_per_file, generator=g) < 0.03).float().numpy())}
        for j in range(num_dense):
            cols[f"d{j}"] = pa.array(torch.randn(rows_per_file, generator=g).abs().log1p().numpy())
        for j in range(num_sparse):
            lens = torch.randint(1, max_bag + 1, (rows_per_file,), generator=g).numpy()
            offs = np.zeros(rows_per_file + 1, dtype=np.int32)
            np.cumsum(lens, out=offs[1:])
            ids = zipf_ids(int(offs[-1]), vocab, 1.05, g).numpy()
            cols[f"s{j}"] = pa.ListArray.from_arrays(pa.array(offs), pa.array(ids))
        path = os.path.join(directory, f"part-{k:05d}.parquet")
        pq.write_table(pa.table(cols), path, row_group_size=row_group)
        paths.append(path)
    return paths


# ----------------------------------------------------------------- runner
_END = object()


def run_throughput_benchmark(paths: Sequence[str], *, input_workers: int = 2, reader_workers: int = 4,
                             samples_per_input_step: int = 4096, steps: int = 20, num_sparse: int = 26,
                             num_dense: int = 13, rows_per_item: int = 4096, dedup: bool = True,
                             queue_depth: int = 4) -> dict[str, Any]:
    """Run the reader -> input -> sink graph until every sink has ``steps`` steps; returns the summary."""
    if reader_workers % input_workers:
        raise ValueError("reader_workers must be a multiple of input_workers")
    factory = ParquetSourceFactory(paths, rows_per_item=rows_per_item)
    items = factory.plan()
    if not items:
        raise ValueError("no work items in the given files")
    feats = [f"s{j}" for j in range(num_sparse)]
    layout = TrainingFeatureLayout(columns={f: f for f in feats} | {f"d{j}": f"d{j}" for j in range(num_dense)},
                                   dense=tuple(f"d{j}" for j in range(num_dense)))
    lanes = [queue.Queue(maxsize=queue_depth) for _ in range(reader_workers)]
    stop = threading.Event()
    errors: list[BaseException] = []
    sinks = [ThroughputSink(r, input_workers, max_steps=steps) for r in range(input_workers)]

    def reader(lane: int) -> None:
        session = factory.create_session()
        try:
            k = lane
            while not stop.is_set():  # cycle the lane's items until the sinks are done
                chunk = session.read(items[k % len(items)])
                k += reader_workers
                while not stop.is_set():
                    try:
                        lanes[lane].put(chunk, timeout=0.1)
                        break
                    except queue.Full:
                        continue
        except BaseException as exc:  # noqa: BLE001 - surfaced by the runner
            errors.append(exc)
            stop.set()
        finally:
            session.close()

    def input_rank(rank: int) -> None:
        factor = reader_workers // input_workers
        my_lanes = [rank * factor + j for j in range(factor)]
        asm = BatchAssembler(samples_per_input_step, "pad")
        sink = sinks[rank]
        j = 0
        try:
            while not sink.done and not stop.is_set():
                try:
                    chunk = lanes[my_lanes[j % factor]].get(timeout=0.1)
                except queue.Empty:
                    continue
                j += 1
                for batch in asm.push(chunk):
                    td = table_to_training_dict(batch.data, layout, sparse_groups={"ids": feats},
                                                label_column="label")
                    if dedup:
                        unique_first_occurrence(torch.from_numpy(td.sparse["ids"][1]))
                    sink.consume(batch.validity.valid_count)
                    if sink.done:
                        break
        except BaseException as exc:  # noqa: BLE001
            errors.append(exc)
            stop.set()

    threads = [threading.Thread(target=reader, args=(i,), daemon=True) for i in range(reader_workers)]
    inputs = [threading.Thread(target=input_rank, args=(r,), daemon=True) for r in range(input_workers)]
    t0 = time.perf_counter()
    for t in threads + inputs:
        t.start()
    for t in inputs:
        t.join()
    wall = time.perf_counter() - t0
    stop.set()
    for t in threads:
        t.join(timeout=5)
    if errors:
        raise errors[0]
    return summarize_sink_reports([s.report() for s in sinks], input_workers=input_workers,
                                  reader_workers=reader_workers, samples_per_input_step=samples_per_input_step,
                                  global_batch_size=samples_per_input_step * input_workers, steps=steps,
                                  wall_seconds=wall)


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--paths", nargs="*", default=None, help="Parquet files (default: synthetic files in a temp dir)")
    p.add_argument("--input-workers", type=int, default=2)
    p.add_argument("--reader-workers", type=int, default=4)
    p.add_argument("--samples-per-input-step", type=int, default=4096)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--rows-per-file", type=int, default=65536)
    p.add_argument("--no-dedup", action="store_true")
    args = p.parse_args(argv)
    with tempfile.TemporaryDirectory() as tmp:
        paths = args.paths or write_synthetic_parquet(tmp, rows_per_file=args.rows_per_file)
        summary = run_throughput_benchmark(paths, input_workers=args.input_workers,
                                           reader_workers=args.reader_workers,
                                           samples_per_input_step=args.samples_per_input_step, steps=args.steps,
                                           dedup=not args.no_dedup)
    print(json.dumps(summary), flush=True)


if __name__ == "__main__":
    main()
