"""Multitask ranking recipe: sparse features -> shared MLP -> PLE experts -> per-task towers.

An application of the recipe API on the fused path: the builder declares
the sparse tables and returns an ordinary ``nn.Module`` built from the layer
library (``MLP`` and ``PLE``, whose linear layers are tcgen05 ``TcLinear``);
``RankingModelTrainer`` runs it with the fused embedding collection and the
flat fused optimizer.  Widths default to multiples of 16 so every linear
layer (experts, gates, towers) runs on the tcgen05 GEMM.

Reference shape of such a recipe: recipes/recsys/ranking/recipe.py:22-30
(``model_builder`` / ``ranking_task``) with the PLE / CGC layers of
src/flare/jax/layers/multitask.py:11-170.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn

from ..data.synthetic import synthetic_ranking_batch
from ..models.layers import MLP, PLE
from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from .ranking import BaseRankingRecipe, MultiTargetCrossEntropyLoss, RankingTask

LABELS = {"neg": 0, "click": 1, "like": 2}
TARGETS = ("click", "like")


class LogitHeads(nn.Module):
    """One logit per task: the dot product of the task's tower output with its weight vector."""

    def __init__(self, n_tasks: int, width: int):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(n_tasks, width) * (1.0 / width) ** 0.5)
        self.bias = nn.Parameter(torch.zeros(n_tasks))

    def forward(self, towers: list[torch.Tensor]) -> torch.Tensor:
        h = torch.stack(towers, 1).float()                     # [B, T, W]
        return (h * self.weight.float()).sum(-1) + self.bias.float()


class MultitaskRankingModel(nn.Module):
    def __init__(self, num_dense: int, emb_total: int, *, shared: int = 256, experts: int = 8,
                 expert_width: int = 128, tower: int = 64, n_tasks: int = 2):
        super().__init__()
        self.n_tasks = n_tasks
        self.shared = MLP(num_dense + emb_total, [shared])
        self.ple = PLE(shared, shared, experts, [expert_width], n_tasks + 1)
        self.towers = nn.ModuleList(MLP(expert_width, [tower]) for _ in range(n_tasks))
        self.heads = LogitHeads(n_tasks, tower)

    def forward(self, dense: torch.Tensor, pooled: torch.Tensor, tables: dict) -> torch.Tensor:
        x = torch.cat([dense, pooled.to(dense.dtype)], 1)
        h = self.shared(x)
        outs = self.ple([h] * (self.n_tasks + 1), h)
        return self.heads([tw(o.to(h.dtype)) for tw, o in zip(self.towers, outs[:self.n_tasks])])


@dataclass
class MultitaskModelBuilder:
    vocabs: tuple[int, ...] = (1000, 5000, 20000, 300)
    embedding_dim: int = 32
    num_dense: int = 16
    max_bag_size: int = 8
    sparse_optimizer: SparseOptimizerConfig = field(
        default_factory=lambda: SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05))
    shared: int = 256
    experts: int = 8
    expert_width: int = 128
    tower: int = 64

    def sparse_tables(self) -> list[SparseTableSpec]:
        return [SparseTableSpec(f"f{i}", v, self.embedding_dim, optimizer=self.sparse_optimizer, feature=f"f{i}")
                for i, v in enumerate(self.vocabs)]

    def create_module(self) -> nn.Module:
        return MultitaskRankingModel(self.num_dense, self.embedding_dim * len(self.vocabs), shared=self.shared,
                                     experts=self.experts, expert_width=self.expert_width, tower=self.tower,
                                     n_tasks=len(TARGETS))


def multitask_objective() -> MultiTargetCrossEntropyLoss:
    """click: positive for click and like; like: positive for like only (negatives weigh 1)."""
    return MultiTargetCrossEntropyLoss.create(
        {"click": {"sample_weight": {"neg": -1.0, "click": 1.0, "like": 1.0}},
         "like": {"sample_weight": {"neg": -1.0, "click": -1.0, "like": 1.0}}},
        LABELS, target_names=TARGETS)


@dataclass(frozen=True)
class MultitaskRankingRecipe(BaseRankingRecipe):
    builder: MultitaskModelBuilder = field(default_factory=MultitaskModelBuilder)

    def model_builder(self) -> MultitaskModelBuilder:
        return self.builder

    def ranking_task(self) -> RankingTask:
        return RankingTask(label_column="label", group_id_column="user_id", objective=multitask_objective())


def synthetic_multitask_batch(B: int, vocabs, num_dense: int, max_bag: int, *, seed: int, device=None,
                              n_labels: int = 3):
    """(dense, label ids, offsets, values) of ``data.synthetic.synthetic_ranking_batch`` (labels neg / click /
    like by default)."""
    return synthetic_ranking_batch(B, vocabs, num_dense, max_bag, seed=seed, device=device, n_labels=n_labels)


def make_recipe(batch_size: int = 4096) -> MultitaskRankingRecipe:
    """The multitask recipe with the default builder (the command line's ``--recipe`` factory)."""
    return MultitaskRankingRecipe(name="multitask", task_name="ranking", batch_size=batch_size,
                                  builder=MultitaskModelBuilder())


__all__ = ["LogitHeads", "MultitaskModelBuilder", "MultitaskRankingModel", "MultitaskRankingRecipe",
           "make_recipe", "multitask_objective", "synthetic_multitask_batch"]


def main(argv=None) -> int:
    """Train the multitask recipe on synthetic data (one rank per GPU under torch.distributed.run)."""
    import argparse

    from ..parallel.dist import init_distributed

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch-size", type=int, default=4096, help="per rank")
    ap.add_argument("--no-graph", action="store_true")
    args = ap.parse_args(argv)
    info = init_distributed(timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    builder = MultitaskModelBuilder()
    recipe = MultitaskRankingRecipe(name="multitask", task_name="ranking", batch_size=args.batch_size,
                                    builder=builder)
    tr = recipe.trainer(rank=info.rank, world_size=max(info.world_size, 1), device=dev,
                        use_graph=not args.no_graph, seed=0)
    for s in range(args.steps):
        b = synthetic_multitask_batch(args.batch_size, builder.vocabs, builder.num_dense, builder.max_bag_size,
                                      seed=1000 * info.rank + s, device=dev)
        res = tr.train_step(*b)
        if info.rank == 0 and (s % 5 == 0 or s == args.steps - 1):
            print(f"step {res.step} loss {res.loss:.5f}", flush=True)
    tr.check()
    tr.close()
    if info.world_size > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
