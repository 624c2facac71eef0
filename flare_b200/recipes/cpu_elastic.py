"""Elastic CPU-configuration worker for ``runtime.elastic.run_elastic``.

The global batch stays fixed; each rank trains ``global_batch / world`` of
it with table-wise sharded tables (gloo all-to-all) and all-reduced dense
gradients.  Every ``save_every`` steps the ranks write a checkpoint (every
rank its tables, rank 0 the dense state) into ``steps/<step>.partial`` and
rank 0 renames it to ``steps/<step>`` after a barrier, so only complete
checkpoints are seen; a start at any world size loads the union of the saved
ranks' tables (each table whole at its owner) and skips the batches already
trained.  ``fail_at=(rank, step)`` injects a host-side failure: that rank
raises before training the step.
"""
from __future__ import annotations

import json
import os
import shutil
from pathlib import Path
from typing import Any

import torch

def _latest_committed(root: Path) -> int | None:
    steps = [int(p.name) for p in (root / "steps").glob("*") if p.name.isdigit()]
    return max(steps) if steps else None


def elastic_cpu_worker(rank: int, world: int, root: str, total_steps: int, global_batch: int, seed: int,
                       save_every: int, fail_at: tuple[int, int] | None = None) -> dict[str, Any]:
    import torch.distributed as dist
    import torch.nn as nn

    from .cpu_small import SmallDense, small_tables
    from ..data.synthetic import SmallSyntheticData
    from ..sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection, slice_samples
    from ..sparse.reference import CpuEmbeddingBagCollection
    from ..training.contracts import TrainingExecutionPlan
    from ..training.engine import TrainEngine
    from ..training.flat import DenseOptimizerConfig

    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not divide over {world} ranks")
    B = global_batch // world
    root_p = Path(root)
    torch.manual_seed(seed)
    data = SmallSyntheticData(global_batch, seed=seed)
    init = CpuEmbeddingBagCollection(small_tables(), global_batch, seed=seed).weights
    emb = ShardedCpuEmbeddingBagCollection(small_tables(), B, seed=seed, weights=init)
    model = SmallDense()
    engine = TrainEngine(model, lambda out, y: nn.functional.binary_cross_entropy_with_logits(out, y),
                         TrainingExecutionPlan.replicated(), DenseOptimizerConfig(kind="adam", learning_rate=1e-3),
                         device=torch.device("cpu"))
    start = _latest_committed(root_p) or 0
    if start:
        d = root_p / "steps" / str(start)
        meta = json.loads((d / "meta.json").read_text())
        engine.restore_checkpoint_state(torch.load(d / "dense.pt", weights_only=False))
        emb.load_state_dict([torch.load(d / f"sparse-rank{r}.pt", weights_only=False) for r in range(meta["world"])])
        for _ in range(start):
            data.next()
    lo, hi = rank * B, (rank + 1) * B
    losses = {}
    for step in range(start + 1, total_steps + 1):
        if fail_at is not None and (rank, step) == tuple(fail_at):
            raise RuntimeError(f"injected failure on rank {rank} before step {step}")
        b = data.next()
        emb.set_input(*slice_samples(b.offsets, b.values, data.F, global_batch, lo, hi))
        pooled = emb.forward().requires_grad_(True)
        res = engine.micro_step_once((b.dense[lo:hi], pooled), b.labels[lo:hi])
        emb.backward(engine.input_gradients({"pooled": pooled})["pooled"])
        losses[step] = float(res.loss)
        if save_every and step % save_every == 0:
            part = root_p / "steps" / f"{step}.partial"
            if rank == 0:
                if part.exists():
                    shutil.rmtree(part)
                part.mkdir(parents=True)
            dist.barrier()
            torch.save(emb.state_dict(), part / f"sparse-rank{rank}.pt")
            if rank == 0:
                torch.save(engine.capture_checkpoint_state(), part / "dense.pt")
                (part / "meta.json").write_text(json.dumps({"step": step, "world": world}))
            dist.barrier()
            if rank == 0:
                os.replace(part, root_p / "steps" / str(step))  # the commit: complete or absent
            dist.barrier()
    return {"rank": rank, "world": world, "start": start, "losses": losses, "sparse": emb.state_dict(),
            "dense": engine.capture_checkpoint_state()}


__all__ = ["elastic_cpu_worker"]
