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

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any, Protocol

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


# ------------------------------------------------------------------ contracts
# Spec and record types with the reference's fields (src/flare/training/components/rl/contracts.py:9-40,
# buffer.py:10-30): configuration and data a user writes.
@dataclass(frozen=True)
class ActionSpec:
    shape: tuple[int, ...]
    dtype: str = "int32"
    num_actions: int | None = None


@dataclass(frozen=True)
class RewardSpec:
    shape: tuple[int, ...] = (1,)
    dtype: str = "float32"


@dataclass(frozen=True)
class Experience:
    observations: Mapping[str, Any]
    actions: Any
    rewards: Any
    next_observations: Mapping[str, Any]
    dones: Any
    log_probs: Any | None = None
    values: Any | None = None


@dataclass(frozen=True)
class Trajectory:
    experiences: tuple[Experience, ...]
    total_reward: float
    length: int


@dataclass(frozen=True)
class ReplayBufferSpec:
    capacity: int
    batch_size: int
    prioritized: bool = False
    alpha: float = 0.6
    beta: float = 0.4


@dataclass(frozen=True)
class RolloutBufferSpec:
    buffer_size: int
    gamma: float = 0.99
    gae_lambda: float = 0.95


class BufferProtocol(Protocol):
    def push(self, experience: Experience) -> None: ...
    def sample(self, batch_size: int) -> tuple[Any, ...]: ...
    def size(self) -> int: ...


# ------------------------------------------------------------------ buffers
class ReplayBuffer:
    """Ring buffer of experiences with uniform or proportional prioritized sampling.

    Prioritized mode (Schaul et al. 2016, proportional variant): experience i is drawn with
    probability p_i^alpha / sum_j p_j^alpha, new experiences get the largest priority seen so far,
    and ``sample`` also returns importance weights (N * P(i))^-beta normalised by their maximum;
    ``update_priorities`` sets p_i = |td error| + eps after a learning step."""

    def __init__(self, spec: ReplayBufferSpec, seed: int = 0, eps: float = 1e-6):
        if spec.capacity < 1 or spec.batch_size < 1:
            raise ValueError("capacity and batch_size must be positive")
        self.spec, self.eps = spec, eps
        self.items: list[Experience | None] = [None] * spec.capacity
        self.prio = np.zeros(spec.capacity, dtype=np.float64)
        self.next, self.count = 0, 0
        self.rng = np.random.default_rng(seed)

    def push(self, experience: Experience) -> None:
        self.items[self.next] = experience
        self.prio[self.next] = self.prio[:self.count].max() if self.count else 1.0
        self.next = (self.next + 1) % self.spec.capacity
        self.count = min(self.count + 1, self.spec.capacity)

    def size(self) -> int:
        return self.count

    def sample(self, batch_size: int | None = None) -> tuple[list[Experience], np.ndarray, np.ndarray]:
        """(experiences, indices, importance weights) of a batch (uniform: weights are 1)."""
        n = batch_size or self.spec.batch_size
        if self.count == 0:
            raise ValueError("the buffer is empty")
        if self.spec.prioritized:
            p = self.prio[:self.count] ** self.spec.alpha
            p = p / p.sum()
            idx = self.rng.choice(self.count, size=n, p=p)
            w = (self.count * p[idx]) ** (-self.spec.beta)
            w = w / w.max()
        else:
            idx = self.rng.integers(0, self.count, size=n)
            w = np.ones(n)
        return [self.items[i] for i in idx], idx, w

    def update_priorities(self, indices, td_errors) -> None:
        self.prio[np.asarray(indices)] = np.abs(np.asarray(td_errors, dtype=np.float64)) + self.eps


class RolloutBuffer:
    """On-policy rollout of ``buffer_size`` steps; ``finish`` computes GAE advantages and returns."""

    def __init__(self, spec: RolloutBufferSpec):
        self.spec = spec
        self.experiences: list[Experience] = []
        self.advantages = self.returns = None

    def push(self, experience: Experience) -> None:
        if len(self.experiences) >= self.spec.buffer_size:
            raise ValueError("the rollout is full; call finish() and reset()")
        if experience.values is None:
            raise ValueError("a rollout experience needs its value estimate")
        self.experiences.append(experience)

    def size(self) -> int:
        return len(self.experiences)

    def finish(self, next_value=0.0):
        """(advantages, returns) over the stored steps, stacked along time."""
        ex = self.experiences
        stack = lambda xs: torch.stack([torch.as_tensor(x, dtype=torch.float32) for x in xs])  # noqa: E731
        self.advantages, self.returns = compute_gae(stack([e.rewards for e in ex]), stack([e.values for e in ex]),
                                                    stack([e.dones for e in ex]), next_value, self.spec.gamma,
                                                    self.spec.gae_lambda)
        return self.advantages, self.returns

    def sample(self, batch_size: int) -> tuple[list[Experience], torch.Tensor, torch.Tensor]:
        if self.advantages is None:
            raise RuntimeError("call finish() before sampling a rollout")
        idx = torch.randperm(len(self.experiences))[:batch_size]
        return [self.experiences[i] for i in idx.tolist()], self.advantages[idx], self.returns[idx]

    def reset(self) -> None:
        self.experiences.clear()
        self.advantages = self.returns = None


__all__ = ["ActionSpec", "BufferProtocol", "Experience", "ReplayBuffer", "ReplayBufferSpec", "RewardSpec",
           "RolloutBuffer", "RolloutBufferSpec", "Trajectory", "compute_discounted_returns", "compute_gae"]
