"""Ranking recipe API: objective, loss adapter, task and recipe base class.

Keeps the reference's public recipe contracts (recipes/recsys/ranking/
losses.py:13-95, graph/losses.py:7-40, task.py:25-60, recipe.py:22-30):

* ``MultiTargetCrossEntropyLoss.create(sample_weight_map, label_map,
  target_names=...)`` maps each multi-class label id to a per-target binary
  label and weight; the loss is the class- and sample-weighted sum of sigmoid
  BCE over targets, divided by the number of valid rows when a mask is given;
* ``RankingLossAdapter`` turns the global valid-row prefix into sample-mean
  weights ``valid * world_size / valid_count`` so that averaging gradients
  over ranks yields sum(sample gradients) / valid_count;
* ``RankingTask`` binds the label / group-id columns to the objective;
* ``BaseRankingRecipe`` is the application adapter (``model_builder``,
  ``ranking_task``).
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
import torch.nn.functional as F


@dataclass
class MultiTargetCrossEntropyLoss:
    target_labels: np.ndarray   # [targets, labels] 0/1
    target_weights: np.ndarray  # [targets, labels] |weight|
    class_weights: np.ndarray   # [targets]
    targets: tuple[str, ...]

    @classmethod
    def create(cls, sample_weight_map: Mapping[str, Any], label_map: Mapping[str, int], *,
               target_names: tuple[str, ...]) -> "MultiTargetCrossEntropyLoss":
        if not label_map or set(label_map.values()) != set(range(len(label_map))):
            raise ValueError("label indexes must be distinct and contiguous from zero")
        if any(type(i) is not int for i in label_map.values()):
            raise TypeError("label indexes must be integers")
        if not target_names or any(not isinstance(n, str) or not n for n in target_names):
            raise ValueError("target_names must contain non-empty target names")
        if len(set(target_names)) != len(target_names) or set(target_names) != set(sample_weight_map):
            raise ValueError("target_names must cover the weight configuration exactly once")
        n_lab, targets = len(label_map), tuple(target_names)
        labels = np.zeros((len(targets), n_lab), dtype=np.float32)
        weights = np.zeros((len(targets), n_lab), dtype=np.float32)
        cw = np.zeros((len(targets),), dtype=np.float32)
        for ti, t in enumerate(targets):
            cfg = sample_weight_map[t]
            c = cfg.get("class_weight", 1.0)
            if not math.isfinite(c):
                raise ValueError(f"Class weight for '{t}' must be finite.")
            cw[ti] = c
            for lab, w in cfg["sample_weight"].items():
                if lab not in label_map:
                    raise KeyError(f"label '{lab}' not found in label_map.")
                if not math.isfinite(w):
                    raise ValueError(f"Weight for '{lab}' must be finite.")
                labels[ti, label_map[lab]] = float(w > 0)
                weights[ti, label_map[lab]] = abs(float(w))
        return cls(labels, weights, cw, targets)

    def _tables(self, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The label / weight tables on ``dev``, copied there once (later calls make no host transfer,
        so a step that uses the loss can be captured in a CUDA graph after one eager call)."""
        cache = self.__dict__.setdefault("_device_tables", {})
        key = str(dev)
        if key not in cache:
            cache[key] = tuple(torch.as_tensor(a, device=dev)
                               for a in (self.target_labels, self.target_weights, self.class_weights))
        return cache[key]

    def per_target(self, label_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(labels [B,T], weights [B,T]) for integer label ids [B]."""
        lab_t, w_t, cw = self._tables(label_ids.device)
        idx = label_ids.long()
        return lab_t[:, idx].t(), w_t[:, idx].t() * cw

    def __call__(self, logits: torch.Tensor, label_ids: torch.Tensor, row_weights: torch.Tensor,
                 valid_mask: torch.Tensor | None = None) -> torch.Tensor:
        if row_weights.dim() != 1 or row_weights.shape[0] != logits.shape[0]:
            raise ValueError("row_weights must be a vector aligned with logits")
        labels, weights = self.per_target(label_ids)
        loss = F.binary_cross_entropy_with_logits(logits.float(), labels, reduction="none") * weights
        if valid_mask is not None:
            if valid_mask.dim() != 1 or valid_mask.shape[0] != logits.shape[0]:
                raise ValueError("valid_mask must be a 1D vector aligned with logits")
            mask = valid_mask.float()
            return (loss.sum(-1) * row_weights * mask).sum() / mask.sum().clamp_min(1.0)
        return (loss.sum(-1) * row_weights).sum()


class RankingLossAdapter:
    """Sample-mean weights from the global valid-row prefix."""

    def __init__(self, base_loss_fn: Callable[..., torch.Tensor]):
        if not callable(base_loss_fn):
            raise TypeError("base_loss_fn must be callable")
        self.base_loss_fn = base_loss_fn

    def __call__(self, predictions: Mapping[str, Any], targets: Mapping[str, Any]) -> torch.Tensor:
        logits = predictions["logits"]
        labels = targets["labels"]
        valid_count = torch.as_tensor(targets["samples_valid_count"]).reshape(-1)
        row_start = int(targets["global_row_start"])
        world = int(targets["world_size"])
        if logits.dim() != 2 or labels.dim() != 1 or labels.shape[0] != logits.shape[0]:
            raise ValueError("ranking logits and labels must be row-aligned")
        if valid_count.numel() != 1:
            raise ValueError("ranking validity field has invalid shape")
        rows = row_start + torch.arange(logits.shape[0], device=logits.device)
        valid = (rows < int(valid_count[0])).to(logits.dtype)
        weights = valid * world / float(valid_count[0])
        return self.base_loss_fn(logits, labels, weights)


@dataclass(frozen=True)
class RankingTask:
    label_column: str
    group_id_column: str
    objective: MultiTargetCrossEntropyLoss

    def __post_init__(self) -> None:
        for name in ("label_column", "group_id_column"):
            if not isinstance(getattr(self, name), str) or not getattr(self, name):
                raise ValueError(f"{name} must be a non-empty string")
        if self.label_column == self.group_id_column:
            raise ValueError("label and group ID columns must be distinct")
        if not callable(self.objective):
            raise TypeError("ranking objective must be callable")
        lab = np.asarray(self.objective.target_labels)
        t = self.objective.targets
        if not t or len(set(t)) != len(t):
            raise ValueError("ranking objective must define distinct targets")
        if lab.ndim != 2 or lab.shape[0] != len(t) or not lab.shape[1]:
            raise ValueError("target_labels must have one row per target and label columns")
        if not np.all((lab == 0) | (lab == 1)):
            raise ValueError("target_labels must be binary")


@dataclass(frozen=True)
class BaseRankingRecipe(ABC):
    """Application adapter: supplies the model builder and the ranking task."""

    name: str
    task_name: str
    batch_size: int = 4096
    pipeline_depth: int = 2

    @abstractmethod
    def model_builder(self) -> Any: ...

    @abstractmethod
    def ranking_task(self) -> RankingTask: ...

    def model(self) -> Any:
        """The dense module of the application (``model_builder().create_module()``)."""
        return self.model_builder().create_module()

    def trainer(self, *, rank: int = 0, world_size: int = 1, device=None, use_graph: bool = True, seed: int = 0,
                **kwargs) -> Any:
        """A ``RankingModelTrainer`` for this recipe: the builder's sparse tables on the fused sharded
        collection, its module on the flat fused optimizer, the task's objective as the loss."""
        from ..training.ranking_trainer import RankingModelTrainer

        return RankingModelTrainer(self.model_builder(), self.ranking_task().objective, self.batch_size, rank=rank,
                                   world_size=world_size, device=device, use_graph=use_graph, seed=seed, **kwargs)


__all__ = ["BaseRankingRecipe", "MultiTargetCrossEntropyLoss", "RankingLossAdapter", "RankingTask"]
