"""The synthetic CPU ranking configuration (single process, fp32).

13 dense N(0,1) features, 8 single-id categorical features (Zipf(1.1) over
1,000 ids per table), embedding dim 16 with sum pooling, bottom MLP
13-64-16 with ReLU, pairwise dot interaction over the 9 vectors, top MLP
52-64-32-1, Bernoulli(sigmoid(a.x + 0.5 N(0,1))) labels; row-wise Adagrad
(lr 0.01) for the tables and Adam (lr 1e-3) for the dense weights; batch 256,
200 steps.  Dense training goes through ``TrainEngine`` (world size 1 or a
gloo group) and the tables through the CPU reference collection, the same
forward/backward contract as the fused GPU collection.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from ..data.synthetic import SmallSyntheticData
from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from ..sparse.reference import CpuEmbeddingBagCollection
from ..training.contracts import TrainingExecutionPlan
from ..training.engine import TrainEngine
from ..training.flat import DenseOptimizerConfig


class DotInteraction(nn.Module):
    def __init__(self, num_vectors: int):
        super().__init__()
        ii, jj = torch.tril_indices(num_vectors, num_vectors, offset=-1)
        self.register_buffer("ii", ii, persistent=False)
        self.register_buffer("jj", jj, persistent=False)

    def forward(self, bot: torch.Tensor, emb: torch.Tensor) -> torch.Tensor:
        z = torch.cat([bot.unsqueeze(1), emb], 1)
        zz = torch.bmm(z, z.transpose(1, 2))
        return torch.cat([bot, zz[:, self.ii, self.jj]], 1)


class SmallDense(nn.Module):
    def __init__(self, num_dense: int = 13, num_sparse: int = 8, dim: int = 16):
        super().__init__()
        self.F, self.D = num_sparse, dim
        self.bottom = nn.Sequential(nn.Linear(num_dense, 64), nn.ReLU(), nn.Linear(64, dim), nn.ReLU())
        self.inter = DotInteraction(num_sparse + 1)
        width = dim + (num_sparse + 1) * num_sparse // 2
        self.top = nn.Sequential(nn.Linear(width, 64), nn.ReLU(), nn.Linear(64, 32), nn.ReLU(), nn.Linear(32, 1))

    def forward(self, inputs):
        dense, pooled = inputs
        bot = self.bottom(dense)
        x = self.inter(bot, pooled.reshape(-1, self.F, self.D))
        return self.top(x)


@dataclass
class SmallRunResult:
    losses: list[float]
    samples_per_s: float
    steps: int
    windows: list = field(default_factory=list)  # flushed metric windows (train/auc_ctr, loss, throughput)


def small_tables(opt: SparseOptimizerConfig | None = None) -> list[SparseTableSpec]:
    opt = opt or SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.01)
    return [SparseTableSpec(f"c{i}", 1000, 16, optimizer=opt) for i in range(8)]


def train_small_cpu(steps: int = 200, batch_size: int = 256, seed: int = 0, storage=None,
                    native: bool = True, checkpoint_dir: str | None = None, save_every: int = 0,
                    resume: bool = False, metrics_every: int = 50) -> SmallRunResult:
    """``storage`` (``SparseStorageOptions``): keep the tables in the paged store (memory limit, disk
    spill), starting from the same initial rows as the in-memory run.  ``native``: pool and reduce
    the sparse gradients with the host C++ ops (the tensor-op path otherwise).  ``checkpoint_dir``:
    save every ``save_every`` steps (``checkpoint.cpu``); ``resume`` continues from the latest
    complete step (the synthetic stream skips the batches already trained on), so ``steps`` counts
    the steps of this call."""
    torch.manual_seed(seed)
    import torch.distributed as dist

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if world > 1:  # global batch batch_size * world; tables dealt to the ranks (gloo all-to-all)
        return _train_small_sharded(steps, batch_size, seed, native, rank, world, metrics_every)
    data = SmallSyntheticData(batch_size, seed=seed)
    emb = CpuEmbeddingBagCollection(small_tables(), batch_size, seed=seed, native=native)
    if storage is not None:
        emb = CpuEmbeddingBagCollection(small_tables(), batch_size, seed=seed, storage=storage, weights=emb.weights)
    model = SmallDense()
    engine = TrainEngine(model, lambda out, y: nn.functional.binary_cross_entropy_with_logits(out, y),
                         TrainingExecutionPlan.replicated(), DenseOptimizerConfig(kind="adam", learning_rate=1e-3),
                         device=torch.device("cpu"))
    start = 0
    if resume and checkpoint_dir is not None:
        from ..checkpoint.cpu import restore_cpu
        from ..checkpoint.store import latest_step

        if latest_step(checkpoint_dir) is not None:
            start = restore_cpu(checkpoint_dir, engine, emb)
            for _ in range(start):
                data.next()
    from ..metrics.aggregation import TrainMetricsWindow

    window = TrainMetricsWindow(window_steps=metrics_every, capacity=metrics_every * batch_size)
    windows = []
    losses = []
    t0 = time.perf_counter()
    for step in range(start + 1, start + steps + 1):
        b = data.next()
        emb.set_input(b.offsets, b.values)
        pooled = emb.forward().requires_grad_(True)
        res = engine.micro_step_once((b.dense, pooled), b.labels)
        emb.backward(engine.input_gradients({"pooled": pooled})["pooled"])
        losses.append(float(res.loss))
        w = window.update(res.outputs.detach(), b.labels, loss_sum=float(res.loss) * batch_size)
        if w is not None:
            windows.append(w)
        if checkpoint_dir is not None and save_every and step % save_every == 0:
            from ..checkpoint.cpu import save_cpu

            save_cpu(checkpoint_dir, step, engine, emb)
    dt = time.perf_counter() - t0
    return SmallRunResult(losses, steps * batch_size / dt, steps, windows)


def _train_small_sharded(steps: int, batch_size: int, seed: int, native: bool, rank: int, world: int,
                         metrics_every: int = 50) -> SmallRunResult:
    """The same model over ``world`` gloo ranks: each rank trains ``batch_size`` samples of a global batch;
    dense gradients are all-reduced (ZeRO-0), the tables are sharded table-wise; the tables start
    from the single-process run's rows, so the trajectory matches it on the global batch."""
    from ..sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection, slice_samples

    data = SmallSyntheticData(batch_size * world, seed=seed)
    init = CpuEmbeddingBagCollection(small_tables(), batch_size * world, seed=seed).weights
    emb = ShardedCpuEmbeddingBagCollection(small_tables(), batch_size, seed=seed, native=native, weights=init)
    model = SmallDense()
    engine = TrainEngine(model, lambda out, y: nn.functional.binary_cross_entropy_with_logits(out, y),
                         TrainingExecutionPlan.replicated(), DenseOptimizerConfig(kind="adam", learning_rate=1e-3),
                         device=torch.device("cpu"))
    from ..metrics.aggregation import TrainMetricsWindow

    window = TrainMetricsWindow(window_steps=metrics_every, capacity=metrics_every * batch_size)  # merged over ranks
    lo, hi = rank * batch_size, (rank + 1) * batch_size
    losses, windows = [], []
    t0 = time.perf_counter()
    for _ in range(steps):
        b = data.next()
        emb.set_input(*slice_samples(b.offsets, b.values, data.F, batch_size * world, lo, hi))
        pooled = emb.forward().requires_grad_(True)
        res = engine.micro_step_once((b.dense[lo:hi], pooled), b.labels[lo:hi])
        emb.backward(engine.input_gradients({"pooled": pooled})["pooled"])
        losses.append(float(res.loss))
        w = window.update(res.outputs.detach(), b.labels[lo:hi], loss_sum=float(res.loss) * batch_size)
        if w is not None:
            windows.append(w)
    dt = time.perf_counter() - t0
    return SmallRunResult(losses, steps * batch_size * world / dt, steps, windows)


def train_small_oracle(steps: int = 200, batch_size: int = 256, seed: int = 0) -> list[float]:
    """Plain PyTorch oracle: nn.EmbeddingBag weights + torch.optim.Adam + explicit row-wise Adagrad."""
    torch.manual_seed(seed)
    data = SmallSyntheticData(batch_size, seed=seed)
    ref = CpuEmbeddingBagCollection(small_tables(), batch_size, seed=seed)  # same initial tables
    tables = [w.clone().requires_grad_(True) for w in ref.weights]
    state = [torch.zeros(w.shape[0]) for w in tables]
    model = SmallDense()
    opt = torch.optim.Adam(model.parameters(), lr=1e-3, eps=1e-8)
    losses = []
    for _ in range(steps):
        b = data.next()
        offs = b.offsets.long()
        pooled = []
        for f, w in enumerate(tables):
            seg = offs[f * batch_size:(f + 1) * batch_size + 1]
            pooled.append(nn.functional.embedding_bag(b.values[seg[0]:seg[-1]].long(), w,
                                                      seg[:-1] - seg[0], mode="sum"))
        out = model((b.dense, torch.cat(pooled, 1)))
        loss = nn.functional.binary_cross_entropy_with_logits(out, b.labels)
        opt.zero_grad()
        for w in tables:
            w.grad = None
        loss.backward()
        opt.step()
        with torch.no_grad():
            for w, s in zip(tables, state):
                g = w.grad
                rows = torch.nonzero(g.abs().sum(1) > 0).flatten()
                s[rows] += (g[rows] ** 2).mean(1)
                w[rows] -= 0.01 * g[rows] / (torch.sqrt(s[rows]).unsqueeze(1) + 1e-8)
        losses.append(float(loss.detach()))
    return losses


def main(argv=None) -> int:
    """``python -m flare_b200.recipes.cpu_small [--steps N] [--batch B] [--checkpoint-dir D --save-every K]
    [--resume] [--memory-limit BYTES --spill-dir DIR] [--tensor-ops]``: one JSON line (samples/s, losses)."""
    import argparse
    import json

    p = argparse.ArgumentParser(prog="flare_b200.recipes.cpu_small")
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--checkpoint-dir", default=None)
    p.add_argument("--save-every", type=int, default=0)
    p.add_argument("--resume", action="store_true")
    p.add_argument("--memory-limit", type=int, default=None, help="sparse storage memory limit (bytes)")
    p.add_argument("--spill-dir", default=None)
    p.add_argument("--tensor-ops", action="store_true", help="tensor-op sparse step instead of the native one")
    a = p.parse_args(argv)
    storage = None
    if a.memory_limit is not None or a.spill_dir is not None:
        from ..sparse.storage import SparseStorageOptions

        storage = SparseStorageOptions(memory_limit_bytes=a.memory_limit, spill_directory=a.spill_dir)
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():  # launched by torch.distributed.run: gloo ranks
        from ..parallel.dist import init_distributed

        init_distributed(backend="gloo")
    r = train_small_cpu(a.steps, a.batch, a.seed, storage=storage, native=not a.tensor_ops,
                        checkpoint_dir=a.checkpoint_dir, save_every=a.save_every, resume=a.resume)
    rank = dist.get_rank() if dist.is_initialized() else 0
    if dist.is_initialized():
        dist.destroy_process_group()
    if rank != 0:
        return 0
    print(json.dumps({"metric": "train samples/s", "value": r.samples_per_s, "steps": r.steps,
                      "first_loss": r.losses[0] if r.losses else None, "last_loss": r.losses[-1] if r.losses else None,
                      "last_window": r.windows[-1] if r.windows else None,
                      "config": {"batch_per_rank": a.batch, "ranks": world, "tables": 8, "rows_per_table": 1000,
                                 "dim": 16,
                                 "sparse_step": "tensor ops" if a.tensor_ops else "native C++",
                                 "storage": "paged" if storage else "in memory"}}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["SmallDense", "SmallRunResult", "main", "small_tables", "train_small_cpu", "train_small_oracle"]
