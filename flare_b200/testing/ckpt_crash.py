"""Crash-window driver for the checkpoint tests: a CPU model whose save can die mid-way.

    python -m flare_b200.testing.ckpt_crash ROOT first    # steps 1..10, FULL save of step 10
    python -m flare_b200.testing.ckpt_crash ROOT crash    # restore, steps 11..20, die (os._exit(86)) inside the save
    python -m flare_b200.testing.ckpt_crash ROOT resume   # restore the last complete step, redo 11..20, save

The model is the checkpoint layer's real input on the CPU: a ``DenseState``
(flat fp32 master / Adam moments) and an in-memory sparse collection with the
attributes ``save_sparse`` / ``load_sparse`` read (shards, fields, dirty rows,
optimizer step).  The crash is a process exit between the dense and the
sparse part of a save, as the reference's crash-recovery workers do with
``os._exit`` around a commit (data/pipeline/production/publish/tests/
crash_recovery_worker.py:65-69).
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass

import torch

from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from ..training.flat import DenseOptimizerConfig, DenseState, FlatParams

TABLES = [SparseTableSpec(name="t0", num_embeddings=50, embedding_dim=8),
          SparseTableSpec(name="t1", num_embeddings=30, embedding_dim=16)]


@dataclass
class _Shard:
    spec: SparseTableSpec
    row_base: int
    col_begin: int = 0
    row_index: int = 0
    row_shards: int = 1
    slot_map_off: int = -1

    @property
    def ncols(self) -> int:
        return self.spec.embedding_dim

    @property
    def storage_rows(self) -> int:
        return self.spec.num_embeddings

    @property
    def row_slice(self) -> slice:
        return slice(None)


class CpuTables:
    """Whole tables on the CPU with a row-wise Adagrad state and dirty-row tracking."""

    def __init__(self, tables: list[SparseTableSpec], seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.tables, self.optimizer = list(tables), SparseOptimizerConfig(kind="rowwise_adagrad")
        self.shards, base = [], 0
        for t in self.tables:
            self.shards.append(_Shard(t, base))
            base += t.num_embeddings
        self.w = [(torch.rand(t.num_embeddings, t.embedding_dim, generator=g) - 0.5) * 0.02 for t in self.tables]
        self.acc = [torch.zeros(t.num_embeddings) for t in self.tables]
        self.dirty = torch.zeros(base, dtype=torch.uint8)
        self.step = 0
        self.step_dev = torch.zeros(1, dtype=torch.int32)

    def shard_fields(self, i: int) -> dict[str, torch.Tensor]:
        return {"weight": self.w[i], "state_row": self.acc[i]}

    def dirty_rows(self, row_base: int, rows: int) -> torch.Tensor:
        return torch.nonzero(self.dirty[row_base:row_base + rows]).flatten()

    def clear_dirty(self) -> None:
        self.dirty.zero_()

    def load_local_state(self, state: dict) -> None:
        for i, s in enumerate(self.shards):
            st = state[(s.spec.name, s.col_begin, s.row_index)]
            self.w[i].copy_(st["weight"])
            self.acc[i].copy_(st["state_row"])

    def update(self, step: int) -> None:
        """A deterministic stand-in for one sparse step: a few rows change, their state grows."""
        for i, s in enumerate(self.shards):
            rows = torch.tensor([(step * 7 + k * 3) % s.storage_rows for k in range(3)])
            self.w[i][rows] += 0.01 * step
            self.acc[i][rows] += 1.0
            self.dirty[s.row_base + rows] = 1
        self.step += 1


class CpuModel:
    def __init__(self, seed: int = 0):
        params = FlatParams()
        params.register("w", (4, 6), "normal", 0.1)
        params.register("b", (4,), "zeros")
        self.dense = DenseState(params, DenseOptimizerConfig(), device=torch.device("cpu"), seed=seed)
        self.emb = CpuTables(TABLES, seed)

    def run(self, first: int, last: int) -> None:
        entries = list(self.dense.params.entries.values())  # the flat padding is not checkpoint state
        for step in range(first, last + 1):
            for e in entries:
                self.dense.master[e.offset:e.offset + e.numel] += 1e-3 * step
            self.dense.compute.copy_(self.dense.master.to(self.dense.compute.dtype))
            self.dense.step += 1
            self.emb.update(step)

    def digest(self) -> list[float]:
        return [float(self.dense.master.sum()), float(self.dense.step)] + \
               [float(w.sum()) for w in self.emb.w] + [float(a.sum()) for a in self.emb.acc] + [float(self.emb.step)]


def main(argv=None) -> int:
    from ..checkpoint import store

    root, phase = (argv or sys.argv[1:])[:2]
    mgr = store.CheckpointManager(root)
    model = CpuModel()
    if phase == "first":
        model.run(1, 10)
        mgr.save(10, model)
        return 0
    start = mgr.restore(model)
    model.run(start + 1, 20)
    if phase == "crash":
        real = store.save_sparse

        def dying_save_sparse(*args, **kwargs):  # the dense part is on disk, the sparse part is not
            os._exit(86)
            return real(*args, **kwargs)

        store.save_sparse = dying_save_sparse
    mgr.save(20, model, incremental=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
