"""A self-contained ranking example: a linear two-target model trained with SGD on four samples.

``run_synthetic_ranking()`` builds a ``RankingTask`` (label and group-id
columns, a two-target ``MultiTargetCrossEntropyLoss`` whose sample weights
encode each target's label by sign), trains a [features, targets] weight
matrix with plain SGD and returns the initial and final loss and the scores.
It runs on the CPU in well under a second and exercises the recipe contracts
end to end.  Reference counterpart: recipes/recsys/examples/synthetic_ranking.py.

    python -m flare_b200.recipes.examples
"""
from __future__ import annotations

import json
from dataclasses import dataclass

import torch

from .ranking import MultiTargetCrossEntropyLoss, RankingTask


@dataclass(frozen=True)
class SyntheticRankingConfig:
    target_names: tuple[str, ...] = ("engagement", "reply")
    input_width: int = 2
    learning_rate: float = 0.1
    steps: int = 40


def run_synthetic_ranking(config: SyntheticRankingConfig | None = None) -> dict:
    cfg = config or SyntheticRankingConfig()
    task = RankingTask(label_column="outcome", group_id_column="visitor",
                       objective=MultiTargetCrossEntropyLoss.create(
                           {t: {"sample_weight": {"negative": -1.0, "positive": 1.0}} for t in cfg.target_names},
                           {"negative": 0, "positive": 1}, target_names=cfg.target_names))
    x = torch.tensor([[-1.0, -1.0], [-1.0, 0.0], [1.0, 0.0], [1.0, 1.0]])
    labels = torch.tensor([0, 0, 1, 1])
    row_weights = torch.full((4,), 0.25)
    w = torch.zeros(cfg.input_width, len(cfg.target_names), requires_grad=True)
    opt = torch.optim.SGD([w], lr=cfg.learning_rate)

    def loss() -> torch.Tensor:
        return task.objective(x @ w, labels, row_weights)

    with torch.no_grad():
        initial = float(loss())
    for _ in range(cfg.steps):
        opt.zero_grad()
        loss().backward()
        opt.step()
    with torch.no_grad():
        final = float(loss())
        scores = torch.sigmoid(x @ w).tolist()
    return {"target_names": list(task.objective.targets), "initial_loss": initial, "final_loss": final,
            "scores": scores}


if __name__ == "__main__":
    print(json.dumps(run_synthetic_ranking(), indent=2))


__all__ = ["SyntheticRankingConfig", "run_synthetic_ranking"]
