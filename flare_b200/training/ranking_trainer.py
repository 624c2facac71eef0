"""Train a user ranking model on the fused B200 path.

The application supplies a model builder (the reference's
``BaseRankingRecipe.model_builder()``, recipes/recsys/ranking/recipe.py:22-30):

* ``sparse_tables()`` -> the ``SparseTableSpec`` of every sparse feature;
* ``create_module()`` -> an ``nn.Module`` taking ``(dense [B, num_dense],
  pooled [B, total_dim], tables {name: [B, dim]})`` (bf16) and returning
  logits ``[B, targets]``;
* ``num_dense`` and ``max_bag_size``.

``RankingModelTrainer`` builds the sharded embedding collection (fused
all-to-alls over NVLink) behind a ``FusedEmbeddingBag`` layer, binds the
module's parameters to a flat fused optimizer (``FusedDenseParameters``:
tcgen05 gradients written into the flat buffer, fused Adam / fused ZeRO-1
over peer memory), and runs one step as: lookup -> module -> objective ->
autograd backward (the fused sparse update runs in the lookup's backward)
-> fused dense step.  After ``EAGER_STEPS`` eager steps the whole step,
autograd included, is captured in a CUDA graph and replayed.

The loss is the objective over the global batch: row weights ``1 /
global_batch`` make every rank's gradient its share of the global sample
mean, so the fused reduce-scatter (a sum over ranks) yields the global mean
(the sample-mean contract of src/flare/jax/training/steppers.py:32-90 and the
ranking loss adapter).

``accumulation_steps`` n > 1 makes a step one micro-step of a window: dense
gradients add up in the flat buffer, pooled gradients in the collection's
window, and the n-th micro-step applies both optimizers once to the sums
divided by n (``finish_window`` closes a shorter tail window); one CUDA
graph per micro-step position (the reference's micro-step windows,
src/flare/jax/training/engines/distributed.py:1017-1180).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from ..sparse.collection import ShardedEmbeddingBagCollection
from ..sparse.config import SparseOptimizerConfig
from ..sparse.module import FusedEmbeddingBag
from .flat import DenseOptimizerConfig
from .fused_module import FusedDenseParameters


@dataclass
class RankingStepResult:
    loss: float
    step: int


class RankingModelTrainer:
    EAGER_STEPS = 2

    def __init__(self, builder: Any, objective, batch_size: int, *, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, dense_optimizer: DenseOptimizerConfig | None = None,
                 sparse_optimizer: SparseOptimizerConfig | None = None, use_graph: bool = True, seed: int = 0,
                 values_capacity: int | None = None, accumulation_steps: int = 1):
        from ..parallel.symm import SymmetricHeap

        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.B, self.rank, self.world = int(batch_size), rank, world_size
        self.global_B = self.B * world_size
        self.objective = objective
        self.use_graph = use_graph
        self.accum = int(accumulation_steps)
        tables = list(builder.sparse_tables())
        self.num_dense = int(builder.num_dense)
        max_bag = int(builder.max_bag_size)
        torch.manual_seed(seed)
        module = builder.create_module()
        module.to(self.device)
        heap = None
        if world_size > 1:
            exchange = ShardedEmbeddingBagCollection.exchange_bytes(tables, self.B, max_bag, values_capacity,
                                                                    accumulation_steps=self.accum)
            nparam = sum(p.numel() for p in module.parameters() if p.requires_grad)
            heap = SymmetricHeap(exchange + 6 * (nparam + 4096 * world_size) + (64 << 20), rank=rank,
                                 world_size=world_size, device=self.device)
        self.heap = heap
        self.coll = ShardedEmbeddingBagCollection(tables, self.B, max_bag_size=max_bag, rank=rank,
                                                  world_size=world_size, device=self.device, heap=heap,
                                                  optimizer=sparse_optimizer, seed=seed,
                                                  values_capacity=values_capacity, accumulation_steps=self.accum)
        self.emb = FusedEmbeddingBag(self.coll, update="deferred" if self.accum > 1 else "immediate")
        self.module = module
        self.dense = FusedDenseParameters(module, dense_optimizer or DenseOptimizerConfig(), device=self.device,
                                          rank=rank, world_size=world_size, heap=heap)
        bf = dict(dtype=torch.bfloat16, device=self.device)
        self.x_dense = torch.zeros(self.B, self.num_dense, **bf)
        self.label_ids = torch.zeros(self.B, dtype=torch.int64, device=self.device)
        self.row_weights = torch.full((self.B,), 1.0 / self.global_B, device=self.device)
        self.loss = torch.zeros((), device=self.device)
        self.steps = 0
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}  # micro-step position -> graph

    # ------------------------------------------------------------------ step
    def set_batch(self, dense: torch.Tensor, label_ids: torch.Tensor, offsets: torch.Tensor,
                  values: torch.Tensor) -> None:
        self.x_dense.copy_(dense, non_blocking=True)
        self.label_ids.copy_(label_ids.reshape(-1), non_blocking=True)
        self.emb.set_input(offsets, values)

    def _body(self) -> torch.Tensor:
        pooled = self.emb()
        logits = self.module(self.x_dense, pooled, self.emb.split(pooled))
        loss = self.objective(logits, self.label_ids, self.row_weights)
        loss.backward()
        if self.accum == 1:
            self.dense.step()
        elif self.coll.micro_filled == self.accum:
            self._close_window()
        return loss.detach()

    def _close_window(self) -> None:
        micro = self.coll.micro_filled
        self.emb.apply_pending()
        self.dense.step(grad_scale=1.0 / micro)

    def finish_window(self) -> bool:
        """Apply the optimizers to an open (tail) window, normalised by its micro-step count."""
        if self.accum > 1 and self.coll.micro_filled > 0:
            self._close_window()
            return True
        return False

    @property
    def graph(self) -> torch.cuda.CUDAGraph | None:
        """The first captured step (None before capture)."""
        return next(iter(self.graphs.values()))[0] if self.graphs else None

    # host-side mirrors of the device state: capture records kernels without running them, so the
    # mirrors it advanced are put back; a replay advances them as the eager step would
    def _host_state(self) -> tuple:
        return self.dense.state.step, self.coll.step, self.coll.micro_filled, self.coll._micro, self.emb.pending

    def _restore_host_state(self, st: tuple) -> None:
        self.dense.state.step, self.coll.step, self.coll.micro_filled, self.coll._micro, self.emb.pending = st

    def _advance_host_state(self) -> None:
        if self.accum > 1:
            k = self.coll.micro_filled
            self.coll._micro = k
            if k + 1 < self.accum:
                self.coll.micro_filled, self.emb.pending = k + 1, True
                return
            self.coll.micro_filled, self.emb.pending = 0, False
        self.dense.state.step += 1
        self.coll.step += 1

    def _run(self) -> torch.Tensor:
        self.module.train()
        self.emb.train()
        if self.use_graph and self.steps >= self.EAGER_STEPS:
            key = self.coll.micro_filled
            if key not in self.graphs:
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                st = self._host_state()
                with torch.cuda.graph(g):
                    out = self._body()
                self._restore_host_state(st)
                self.graphs[key] = (g, out)
            g, out = self.graphs[key]
            g.replay()
            self._advance_host_state()
            self.loss.copy_(out)
            return self.loss
        out = self._body()
        self.loss.copy_(out)
        return self.loss

    def train_step(self, dense: torch.Tensor, label_ids: torch.Tensor, offsets: torch.Tensor,
                   values: torch.Tensor) -> RankingStepResult:
        """One step on this rank's batch; returns the global-mean loss contribution of this rank."""
        self.set_batch(dense, label_ids, offsets, values)
        loss = self._run()
        self.steps += 1
        return RankingStepResult(float(loss.item()), self.steps)

    @torch.no_grad()
    def predict(self, dense: torch.Tensor, offsets: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        """Probabilities of a batch; an open accumulation window is applied first."""
        self.finish_window()
        self.module.eval()
        self.emb.eval()
        self.x_dense.copy_(dense)
        self.emb.set_input(offsets, values)
        pooled = self.emb()
        logits = self.module(self.x_dense, pooled, self.emb.split(pooled))
        return torch.sigmoid(logits.float())

    # ------------------------------------------------------------ checkpoints
    def checkpoint_parts(self) -> "_CheckpointParts":
        """What ``checkpoint.store.CheckpointManager`` saves and restores: the flat dense state
        (fp32 master, optimizer moments, step; parameters by name with their logical shapes) and the
        sparse collection (FULL or INCREMENTAL)."""
        return _CheckpointParts(self)

    def save_checkpoint(self, manager, step: int, *, incremental: bool | None = None):
        """Write ``step`` through ``manager``; an open accumulation window is applied first, so a
        checkpoint is always cut at an optimizer boundary."""
        torch.cuda.synchronize(self.device)
        return manager.save(step, self.checkpoint_parts(), incremental=incremental)

    def restore_checkpoint(self, manager, step: int | None = None) -> int:
        """Load ``step`` (the newest committed one by default) in place: captured graphs stay valid."""
        step = manager.restore(self.checkpoint_parts(), step)
        torch.cuda.synchronize(self.device)
        return step

    def check(self) -> None:
        self.coll.check()

    def close(self) -> None:
        self.finish_window()
        self.graphs.clear()


class _CheckpointParts:
    def __init__(self, trainer: RankingModelTrainer):
        self._trainer = trainer
        self.dense = trainer.dense.state
        self.emb = trainer.coll

    def flush_pending_updates(self) -> None:
        self._trainer.finish_window()


__all__ = ["RankingModelTrainer", "RankingStepResult"]
