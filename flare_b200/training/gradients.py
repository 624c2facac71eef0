"""Gradient helpers of the generic engine: window means and the sparse input-gradient contract.

* ``mean_accumulated_gradients``: a window's summed gradients divided by its
  actual micro-step count (a partial window divides by its own length).
* ``normalize_input_gradients``: the sample-mean contract for gradients that
  leave the dense model towards the sparse tables.  Each rank's loss is the
  mean over its own samples, and the dense gradients are averaged over the
  ranks (and the window); the gradients w.r.t. the pooled embeddings are
  divided by ``world_size * micro_steps`` once, so that the sparse update of
  a row equals the one a single rank would make on the global batch.  It
  must not be applied again at the sparse optimizer's commit.
* ``input_gradients``: the gradients autograd left on the inputs that asked
  for them (``requires_grad``), normalised as above.

Reference behaviour: src/flare/jax/training/gradients/normalization.py:11-40
and the input-gradient partition of src/flare/jax/training/steppers.py:32-90.
"""
from __future__ import annotations

from collections.abc import Mapping

import torch


def mean_accumulated_gradients(accumulated, micro_steps: int):
    if micro_steps <= 0:
        raise ValueError(f"micro_steps must be positive, got {micro_steps}")
    if isinstance(accumulated, Mapping):
        return {k: v / micro_steps for k, v in accumulated.items()}
    return accumulated / micro_steps


def normalize_input_gradients(gradients: Mapping[str, torch.Tensor], *, world_size: int,
                              micro_steps: int) -> dict[str, torch.Tensor]:
    if world_size <= 0:
        raise ValueError(f"world_size must be positive, got {world_size}")
    if micro_steps <= 0:
        raise ValueError(f"micro_steps must be positive, got {micro_steps}")
    return {k: v.float() / (world_size * micro_steps) for k, v in gradients.items()}


def input_gradients(inputs: Mapping[str, torch.Tensor], *, world_size: int, micro_steps: int) -> dict[str, torch.Tensor]:
    """Normalised gradients of the named inputs that required them (after ``backward``)."""
    grads = {}
    for k, t in inputs.items():
        if t.requires_grad:
            if t.grad is None:
                raise ValueError(f"input {k!r} required a gradient but has none (was backward run?)")
            grads[k] = t.grad
    return normalize_input_gradients(grads, world_size=world_size, micro_steps=micro_steps)


__all__ = ["input_gradients", "mean_accumulated_gradients", "normalize_input_gradients"]
