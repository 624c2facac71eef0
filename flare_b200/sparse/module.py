"""The fused sharded embedding collection as an autograd-aware ``nn.Module``.

``FusedEmbeddingBag`` wraps a ``ShardedEmbeddingBagCollection`` so that a
user model composes it like any other layer:

* ``set_input(offsets, values)`` stages the keyed-jagged batch;
* ``forward()`` runs the fused forward (ids all-to-all, gather + pool,
  pooled all-to-all over NVLink) and returns the pooled rows ``[B,
  total_dim]`` (bf16) as a graph node; ``split(pooled)`` gives per-table
  views;
* in the backward the pooled gradient is copied into the collection's
  exchange buffer and the fused sparse backward runs at once (pooled-
  gradient all-to-all, dedup, fp32 accumulation, row-wise optimizer), or is
  left for ``apply_pending()`` when ``update="deferred"``.

The gradient contract matches the reference's train worker, which
differentiates the loss with respect to the pooled sparse inputs and sends
them to the table owners (recipes/recsys/ranking/workers/train_worker.py:
271-553; src/flare/jax/training/steppers.py:32-90): the caller's loss
scaling (sample mean over the global batch) is what reaches the tables.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .collection import ShardedEmbeddingBagCollection


class _PooledLookup(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, owner):
        ctx.owner = owner
        pooled = owner.coll.forward(training=owner.training)
        return pooled.view_as(pooled)

    @staticmethod
    def backward(ctx, grad):
        owner = ctx.owner
        owner.coll.grad_input.copy_(grad)
        if owner.update == "immediate":
            owner.coll.backward()
        else:
            owner.pending = True
        return None, None


class FusedEmbeddingBag(nn.Module):
    def __init__(self, coll: ShardedEmbeddingBagCollection, *, update: str = "immediate"):
        super().__init__()
        if update not in ("immediate", "deferred"):
            raise ValueError("update must be 'immediate' or 'deferred'")
        self.coll = coll
        self.update = update
        self.pending = False
        # a leaf that requires grad, so autograd reaches this node's backward
        self.register_buffer("_anchor", torch.zeros(1, device=coll.device, requires_grad=False), persistent=False)
        self._anchor.requires_grad_(True)
        dims, off = [], 0
        for t in coll.tables:
            dims.append((t.name, off, t.embedding_dim))
            off += t.embedding_dim
        self.layout = dims

    @property
    def total_dim(self) -> int:
        return self.coll.total_dim

    def set_input(self, offsets: torch.Tensor, values: torch.Tensor, non_blocking: bool = True) -> None:
        self.coll.set_input(offsets, values, non_blocking=non_blocking)

    def forward(self) -> torch.Tensor:
        if self.training and torch.is_grad_enabled():
            return _PooledLookup.apply(self._anchor, self)
        return self.coll.forward(training=False)

    def split(self, pooled: torch.Tensor) -> dict[str, torch.Tensor]:
        """Per-table views ``name -> [B, dim]`` of a pooled output."""
        return {name: pooled[:, off:off + d] for name, off, d in self.layout}

    def apply_pending(self) -> None:
        """Run the deferred fused sparse backward (``update="deferred"``)."""
        if self.pending:
            self.coll.backward()
            self.pending = False


__all__ = ["FusedEmbeddingBag"]
