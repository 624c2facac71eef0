"""Metric-window latency: exact AUC / GAUC / calibration of a synthetic ranking window.

    python -m flare_b200.benchmarks.metrics [--batches 10] [--rows-per-batch 20000] [--targets 3]
        [--group-cardinality 20000] [--ranks 1,2,4] [--rounds 2] [--device cpu|cuda] [--output out.json]

Measures the metric computation alone, not training: ``batches x rows-per-batch`` rows of random
scores, 0/1 labels (one column per target) and group ids.  Two ways of computing the window:

* ``local``: one process holds every row and computes each target's AUC, GAUC and calibration on
  ``--device`` (the GPU sort kernels for CUDA tensors, the exact CPU reference otherwise);
* for every P in ``--ranks``: P gloo ranks hold an equal share of the rows each and merge them
  exactly (``metrics.distributed.distributed_metrics``: one all-gather of packed (group, score,
  positives, negatives) summaries per target, or with ``--merge partitioned`` groups and score ranges
  split over the ranks), timed between barriers inside the ranks, slowest rank.

Each round visits the rank counts in alternating order so that no rank count always runs first
(cold start); every run must see the same sample count and reach the local values (the merge is
exact, so any difference beyond rounding is an error).  Prints one JSON summary: per way of
computing, the seconds of every round and their median / p50 / p95, and rows per second.

Reference counterpart: tools/validation/benchmark_ranking_metrics.py (the Ray Data metric window at
several parallelisms) and tools/validation/performance_metrics.py (timing summaries).
"""
from __future__ import annotations

import argparse
import json
import math
import time
from pathlib import Path
from statistics import median

import numpy as np
import torch


def quantile(values, q: float) -> float:
    """Linear interpolation between the two order statistics around ``q * (n - 1)``."""
    xs = sorted(float(v) for v in values)
    if not xs:
        raise ValueError("quantile of no values")
    if not 0.0 <= q <= 1.0:
        raise ValueError("q must be in [0, 1]")
    pos = (len(xs) - 1) * q
    lo = int(math.floor(pos))
    hi = min(lo + 1, len(xs) - 1)
    return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)


def timing_summary(seconds, rows: int) -> dict:
    """Median / p50 / p95 of the run times and of ``rows`` per second."""
    secs = [float(s) for s in seconds]
    if not secs or min(secs) <= 0:
        raise ValueError("timings must be positive and non-empty")
    rates = [rows / s for s in secs]
    return {"runs": len(secs), "rows": int(rows), "seconds": secs,
            "elapsed_seconds": {"median": median(secs), "p50": quantile(secs, 0.5), "p95": quantile(secs, 0.95)},
            "rows_per_second": {"median": median(rates), "p50": quantile(rates, 0.5), "p95": quantile(rates, 0.95)}}


def synthetic_window(rows: int, targets: int, group_cardinality: int, seed: int):
    """(scores float32 [rows, targets], labels float32 [rows, targets], groups int64 [rows])."""
    rng = np.random.default_rng(seed)
    scores = rng.random((rows, targets), dtype=np.float32)
    # labels correlated with the scores, so the AUCs are away from 0.5 and a wrong merge shows
    labels = (rng.random((rows, targets), dtype=np.float32) < 0.2 + 0.6 * scores).astype(np.float32)
    groups = rng.integers(0, group_cardinality, rows, dtype=np.int64)
    return scores, labels, groups


def local_metrics(scores: torch.Tensor, labels: torch.Tensor, groups: torch.Tensor) -> dict[str, float]:
    from ..metrics.ranking import auc, calibration, gauc

    out = {}
    for t in range(scores.shape[1]):
        s, y = scores[:, t].contiguous(), labels[:, t].contiguous()
        out[f"auc_{t}"] = auc(s, y)
        out[f"gauc_{t}"] = gauc(s, y, groups)
        out[f"calibration_{t}"] = calibration(s, y)
    return out


def _rank_worker(rank: int, world: int, scores, labels, groups, merge: str = "allgather") -> dict:
    """One rank's share of the window: merge with the others, timed between barriers."""
    import torch.distributed as dist

    from ..metrics.distributed import distributed_metrics

    n = scores.shape[0]
    lo, hi = rank * n // world, (rank + 1) * n // world
    s, y, g = torch.from_numpy(scores[lo:hi]), torch.from_numpy(labels[lo:hi]), torch.from_numpy(groups[lo:hi])
    dist.barrier()
    t0 = time.perf_counter()
    out = {}
    for t in range(s.shape[1]):
        m = distributed_metrics(s[:, t].contiguous(), y[:, t].contiguous(), g, merge=merge)
        for k, v in m.items():
            out[f"{k}_{t}"] = v
    dist.barrier()
    elapsed = time.perf_counter() - t0
    count = torch.tensor([hi - lo], dtype=torch.int64)
    dist.all_reduce(count)
    return {"seconds": elapsed, "samples": int(count.item()), "metrics": out}


def run(*, batches: int = 10, rows_per_batch: int = 20_000, targets: int = 3, group_cardinality: int = 20_000,
        ranks: tuple[int, ...] = (1, 2, 4), rounds: int = 2, device: str = "cpu", seed: int = 1,
        timeout: float = 600.0, merge: str = "allgather") -> dict:
    from ..runtime.launch import spawn_ranks

    counts = (batches, rows_per_batch, targets, group_cardinality, rounds, *ranks)
    if any(int(c) <= 0 for c in counts):
        raise ValueError("batch, row, target, group, round and rank counts must be positive")
    rows = batches * rows_per_batch
    scores, labels, groups = synthetic_window(rows, targets, group_cardinality, seed)
    dev = torch.device(device)
    ts, ty, tg = (torch.from_numpy(a).to(dev) for a in (scores, labels, groups))

    local_secs, ref = [], None
    for _ in range(rounds):
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        ref = local_metrics(ts, ty, tg)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        local_secs.append(time.perf_counter() - t0)

    per_p: dict[int, list[float]] = {p: [] for p in ranks}
    worst = 0.0
    for r in range(rounds):
        for p in (ranks if r % 2 == 0 else tuple(reversed(ranks))):
            res = spawn_ranks(_rank_worker, p, scores, labels, groups, merge, timeout=timeout)
            if any(x["samples"] != rows for x in res):
                raise RuntimeError(f"{p} ranks saw {res[0]['samples']} samples, expected {rows}")
            per_p[p].append(max(x["seconds"] for x in res))
            for k, v in res[0]["metrics"].items():
                if not (math.isnan(v) and math.isnan(ref[k])):
                    worst = max(worst, abs(v - ref[k]))
    if worst > 1e-6:
        raise RuntimeError(f"merged metrics differ from the one-process values by {worst:g}")
    return {
        "samples": rows, "targets": targets, "group_cardinality": group_cardinality, "batches": batches,
        "rounds": rounds, "device": str(dev), "merge": merge,
        "metrics": {k: v for k, v in ref.items()},
        "max_abs_diff_merged_vs_local": worst,
        "local": timing_summary(local_secs, rows),
        "ranks": {str(p): timing_summary(secs, rows) for p, secs in per_p.items()},
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="metric-window latency: exact AUC / GAUC / calibration")
    ap.add_argument("--batches", type=int, default=10)
    ap.add_argument("--rows-per-batch", type=int, default=20_000)
    ap.add_argument("--targets", type=int, default=3)
    ap.add_argument("--group-cardinality", type=int, default=20_000)
    ap.add_argument("--ranks", default="1,2,4", help="comma-separated gloo rank counts")
    ap.add_argument("--rounds", type=int, default=2)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu",
                    help="device of the one-process computation")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--merge", choices=("allgather", "partitioned"), default="allgather",
                    help="how the ranks merge their windows (metrics.distributed.distributed_metrics)")
    ap.add_argument("--output", type=Path)
    args = ap.parse_args(argv)
    summary = run(batches=args.batches, rows_per_batch=args.rows_per_batch, targets=args.targets,
                  group_cardinality=args.group_cardinality, ranks=tuple(int(x) for x in args.ranks.split(",") if x),
                  rounds=args.rounds, device=args.device, seed=args.seed, merge=args.merge)
    text = json.dumps(summary, indent=2)
    if args.output is not None:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(text + "\n")
    print(text, flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
