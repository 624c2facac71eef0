"""Elastic restarts: run a job over ranks; after a rank is lost, restart from the last committed
checkpoint, possibly at another world size.

``run_elastic(worker, world_sizes, *args)`` runs ``worker(rank, world, *args)``
on ``world_sizes[0]`` ranks (``runtime.launch.spawn_ranks``); when a rank
fails (its exception, or its peers' collectives timing out after it left)
the attempt ends and the next one starts on the next world size in the list
(the last one repeats), up to ``max_restarts`` restarts.  The worker is
expected to resume from the newest committed checkpoint it finds, so
training continues from there; everything after that checkpoint is redone.
Returns the final attempt's per-rank results and the log of attempts.

``recipes.cpu_elastic.elastic_cpu_worker`` is such a worker for the CPU configuration: the
global batch stays fixed, each rank trains ``global_batch / world`` of it
with table-wise sharded tables (gloo all-to-all) and all-reduced dense
gradients; every ``save_every`` steps the ranks write a checkpoint (every
rank its tables, rank 0 the dense state) into ``steps/<step>.partial``,
and rank 0 renames it to ``steps/<step>`` after a barrier, so only complete
checkpoints are ever seen; a restart at any world size loads the union of
the saved ranks' tables (each table whole at its owner) and skips the
batches already trained.  ``fail_at=(rank, step)`` injects a host-side
failure: that rank raises before training the step.

Reference behaviour: coordinated checkpoint cut and restore with global
reshard (docs/fluxway_source_adapter.md:109-115, runtime/fluxway/workers/
reader.py:510-516); failures are injected on the host, never on a device.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

from .launch import RankFailure, spawn_ranks


@dataclass
class Attempt:
    world: int
    ok: bool
    seconds: float
    failed_rank: int | None = None
    error: str = ""


@dataclass
class ElasticResult:
    results: list
    attempts: list[Attempt] = field(default_factory=list)


def run_elastic(worker, world_sizes: list[int], *args, max_restarts: int = 3, timeout: float = 300.0,
                pg_timeout_s: float = 10.0) -> ElasticResult:
    if not world_sizes or any(w < 1 for w in world_sizes):
        raise ValueError("world_sizes must list positive world sizes")
    attempts: list[Attempt] = []
    for k in range(max_restarts + 1):
        world = world_sizes[min(k, len(world_sizes) - 1)]
        t0 = time.perf_counter()
        try:
            res = spawn_ranks(worker, world, *args, timeout=timeout, pg_timeout_s=pg_timeout_s)
        except RankFailure as e:
            attempts.append(Attempt(world, False, time.perf_counter() - t0, e.rank, e.detail.strip().splitlines()[-1]))
            continue
        attempts.append(Attempt(world, True, time.perf_counter() - t0))
        return ElasticResult(res, attempts)
    raise RuntimeError(f"the job failed {len(attempts)} times: " + "; ".join(
        f"world {a.world}: rank {a.failed_rank}: {a.error}" for a in attempts))


__all__ = ["Attempt", "ElasticResult", "run_elastic"]
