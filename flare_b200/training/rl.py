"""Advantage estimators for reinforcement-learning fine-tuning of recommenders.

``compute_gae`` (generalised advantage estimation, Schulman et al. 2016) and
``compute_discounted_returns`` work on NumPy arrays or torch tensors (CPU or
CUDA) of shape ``[T]`` or ``[T, N]`` (N parallel environments / users): the
reverse scan runs over time with every environment in one vector op per step,
so a batch of trajectories on the GPU never leaves the device.  ``dones[t]``
marks the end of an episode after step t.  Reference behaviour:
src/flare/training/components/rl/advantages.py:6-60 (single trajectory).
"""
from __future__ import annotations

import numpy as np
import torch


def _as_tensor(x, like=None):
    if isinstance(x, torch.Tensor):
        return x.to(torch.float32)
    dev = like.device if isinstance(like, torch.Tensor) else None
    return torch.as_tensor(np.asarray(x, dtype=np.float32), device=dev)


def compute_gae(rewards, values, dones, next_value=0.0, gamma: float = 0.99, gae_lambda: float = 0.95):
    """(advantages, returns) with returns = advantages + values; same type as ``rewards``."""
    numpy_in = not isinstance(rewards, torch.Tensor)
    r = _as_tensor(rewards)
    v = _as_tensor(values, r)
    d = _as_tensor(dones, r)
    if r.shape != v.shape or r.shape != d.shape:
        raise ValueError("rewards, values and dones must have the same shape")
    nv = _as_tensor(next_value, r).expand(r.shape[1:]) if r.dim() > 1 else _as_tensor(next_value, r).reshape(())
    adv = torch.zeros_like(r)
    last = torch.zeros_like(r[0])
    for t in range(r.shape[0] - 1, -1, -1):
        nxt = nv if t == r.shape[0] - 1 else v[t + 1]
        keep = 1.0 - d[t]
        delta = r[t] + gamma * nxt * keep - v[t]
        last = delta + gamma * gae_lambda * keep * last
        adv[t] = last
    ret = adv + v
    if numpy_in:
        return adv.cpu().numpy(), ret.cpu().numpy()
    return adv, ret


def compute_discounted_returns(rewards, dones, gamma: float = 0.99):
    """Discounted return per step, restarting after every ``done``."""
    numpy_in = not isinstance(rewards, torch.Tensor)
    r = _as_tensor(rewards)
    d = _as_tensor(dones, r)
    out = torch.zeros_like(r)
    run = torch.zeros_like(r[0])
    for t in range(r.shape[0] - 1, -1, -1):
        run = r[t] + gamma * run * (1.0 - d[t])
        out[t] = run
    return out.cpu().numpy() if numpy_in else out


__all__ = ["compute_discounted_returns", "compute_gae"]
