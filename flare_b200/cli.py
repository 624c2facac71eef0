"""Command-line entry points: train and eval of the fused DLRM-family model, and application recipes.

    python -m flare_b200.cli train --model-config model.yaml --batch-per-gpu 8192 --steps 1000 \\
        --checkpoint-dir ckpt --save-every 500 [--data DIR_OF_PARQUET] [--resume]
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m flare_b200.cli train ...
    python -m flare_b200.cli eval --model-config model.yaml --checkpoint-dir ckpt [--step S] --batches 8
    python -m flare_b200.cli recipe --recipe flare_b200.recipes.multitask:make_recipe --steps 100 \
        --checkpoint-dir ckpt --save-every 50 [--resume] [--accumulation-steps 2]

``train`` builds the model from a model-structure file (``{"model": "dlrm",
"tables": [...], ...}``, see ``config.loader.load_model_config``), feeds it
either synthetic batches of the table vocabularies or Parquet files
(``label``, ``d0..``, ``s0..`` list columns) through the prefetching loader,
logs AUC / calibration / loss / throughput windows (console + optional JSONL)
and writes FULL then INCREMENTAL checkpoints.  ``eval`` binds an immutable
checkpoint step as inference weights (verified against its recorded file
evidence), loads it into a one-GPU model and reports AUC / calibration on
held-out batches.  ``recipe`` runs an application recipe (a
``BaseRankingRecipe``: model builder + ranking task) on the fused path:
train on synthetic batches of its tables, checkpoint, resume, and report
per-target AUC.  Reference behaviour: the ranking recipe's train and eval
workers (recipes/recsys/ranking/workers/train_worker.py:271-664, 717-800).
"""
from __future__ import annotations

import argparse
import json
import sys
import time

import torch


def _parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="flare_b200")
    sub = p.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("train")
    t.add_argument("--model-config", required=True)
    t.add_argument("--batch-per-gpu", type=int, default=4096)
    t.add_argument("--steps", type=int, default=100)
    t.add_argument("--max-bag", type=int, default=64)
    t.add_argument("--data", default=None, help="directory or file(s) of Parquet training data")
    t.add_argument("--checkpoint-dir", default=None)
    t.add_argument("--save-every", type=int, default=0)
    t.add_argument("--incremental", action="store_true", help="saves after the first are incremental")
    t.add_argument("--resume", action="store_true")
    t.add_argument("--metrics-every", type=int, default=50)
    t.add_argument("--metrics-jsonl", default=None)
    t.add_argument("--seed", type=int, default=0)
    t.add_argument("--no-graph", action="store_true")
    t.add_argument("--table-shards", default="",
                   help='row-wise pieces per table: "4" (every table) or "t0:4,t3:2" (the rest keep their config)')
    t.add_argument("--sparse-policy", choices=["sync", "pipelined"], default=None,
                   help="default: pipelined when every table allows max_staleness_steps >= 1, else sync")
    t.add_argument("--staleness", type=int, default=None,
                   help="pipelined policy: sparse updates in flight (lookups miss that many steps; default: the "
                        "smallest max_staleness_steps of the tables, at least 1)")
    t.add_argument("--accumulation-steps", type=int, default=1,
                   help="micro-steps per optimizer step (sync policy): sparse and dense updates once per window")
    r = sub.add_parser("recipe", help="train, checkpoint and evaluate an application recipe on the fused path")
    r.add_argument("--recipe", required=True,
                   help="module:attr naming a BaseRankingRecipe, its class, or a factory taking batch_size "
                        "(e.g. flare_b200.recipes.multitask:make_recipe)")
    r.add_argument("--batch-per-gpu", type=int, default=4096)
    r.add_argument("--steps", type=int, default=100)
    r.add_argument("--accumulation-steps", type=int, default=1)
    r.add_argument("--checkpoint-dir", default=None)
    r.add_argument("--save-every", type=int, default=0)
    r.add_argument("--incremental", action="store_true", help="saves after the first are incremental")
    r.add_argument("--resume", action="store_true")
    r.add_argument("--log-every", type=int, default=10)
    r.add_argument("--eval-batches", type=int, default=2, help="held-out synthetic batches per rank after training")
    r.add_argument("--seed", type=int, default=0)
    r.add_argument("--no-graph", action="store_true")
    e = sub.add_parser("eval")
    e.add_argument("--model-config", required=True)
    e.add_argument("--checkpoint-dir", required=True)
    e.add_argument("--step", type=int, default=None)
    e.add_argument("--batch", type=int, default=4096)
    e.add_argument("--batches", type=int, default=8)
    e.add_argument("--max-bag", type=int, default=64)
    e.add_argument("--data", default=None)
    e.add_argument("--seed", type=int, default=12345)
    e.add_argument("--gauc-feature", type=int, default=None,
                   help="also report GAUC, grouping samples by the first id of this sparse feature (e.g. a user id)")
    return p


def _dlrm_cfg(path, table_shards: str = ""):
    from dataclasses import replace

    from .config.loader import load_model_config, parse_group_counts

    name, cfg = load_model_config(path)
    if name != "dlrm":
        raise SystemExit(f"the cli trains the dlrm model family; {name!r} has its own benchmark entry point")
    if table_shards:
        counts = parse_group_counts(table_shards, [t.name for t in cfg.tables], what="table shards")
        cfg.tables = [replace(t, shards=counts.get(t.name, t.shards)) for t in cfg.tables]
    return cfg


def _batches(args, cfg, B, rank, world, device):
    """Iterator of SparseBatch in pinned host memory (Parquet files or synthetic)."""
    if args.data:
        from .data.schema import TrainingFeatureLayout, table_to_training_dict
        from .data.sources import StandardSourceFactory, stream_batches
        from .data.synthetic import SparseBatch

        F, nd = len(cfg.tables), cfg.num_dense
        feats = [f"s{j}" for j in range(F)]
        layout = TrainingFeatureLayout(columns={f: f for f in feats} | {f"d{j}": f"d{j}" for j in range(nd)},
                                       dense=tuple(f"d{j}" for j in range(nd)))
        factory = StandardSourceFactory.create("parquet", {"paths": args.data})
        items = [it for k, it in enumerate(factory.plan()) if k % world == rank]

        def gen():
            while True:
                for ab in stream_batches(factory, B, policy="pad", items=items):
                    td = table_to_training_dict(ab.data, layout, sparse_groups={"ids": feats}, label_column="label")
                    off, vals = td.sparse["ids"]
                    yield SparseBatch(torch.from_numpy(td.dense), torch.from_numpy(td.labels),
                                      torch.from_numpy(off), torch.from_numpy(vals))
        from .data.loader import PrefetchLoader

        return iter(PrefetchLoader(gen(), depth=4))
    from .data.synthetic import DLRMSyntheticData

    gen = DLRMSyntheticData(B, [t.num_embeddings for t in cfg.tables], num_dense=cfg.num_dense,
                            max_bag=args.max_bag, seed=args.seed, rank=rank)

    def syn():
        while True:
            yield gen.next().pin_memory()
    return syn()


def train(args) -> int:
    from .checkpoint.store import CheckpointManager, latest_step
    from .metrics.aggregation import ConsoleSink, JsonlSink, TrainMetricsWindow
    from .parallel.dist import init_distributed, shutdown
    from .training.trainer import DLRMTrainer

    info = init_distributed(timeout_s=300)
    rank, world = info.rank, max(info.world_size, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = _dlrm_cfg(args.model_config, args.table_shards)
    B = args.batch_per_gpu
    trainer = DLRMTrainer(cfg, B, max_bag_size=args.max_bag, rank=rank, world_size=world, device=dev,
                          seed=args.seed, use_graph=not args.no_graph, sparse_policy=args.sparse_policy,
                          staleness=args.staleness, accumulation_steps=args.accumulation_steps)
    mgr = CheckpointManager(args.checkpoint_dir) if args.checkpoint_dir else None
    start = 0
    if args.resume and mgr is not None and latest_step(args.checkpoint_dir) is not None:
        start = mgr.restore(trainer.model)
    sinks = [ConsoleSink()] if rank == 0 else []
    if rank == 0 and args.metrics_jsonl:
        sinks.append(JsonlSink(args.metrics_jsonl))
    window = TrainMetricsWindow(window_steps=args.metrics_every, device=dev, sinks=sinks,
                                capacity=max(args.metrics_every * B, B))
    data = _batches(args, cfg, B, rank, world, dev)
    saved = False
    t0 = time.perf_counter()
    for step in range(start + 1, start + args.steps + 1):
        res = trainer.train_step(next(data))
        window.update(trainer.model.logits, trainer.model.labels, loss_sum=res.loss * B)
        if mgr is not None and args.save_every and step % args.save_every == 0:
            torch.cuda.synchronize(dev)
            mgr.save(step, trainer.model, incremental=args.incremental and saved)
            saved = True
    torch.cuda.synchronize(dev)
    trainer.check()
    if rank == 0:
        dt = time.perf_counter() - t0
        print(json.dumps({"steps": args.steps, "last_step": start + args.steps, "wall_s": dt,
                          "samples_per_s": args.steps * B * world / dt}), flush=True)
    trainer.close()
    shutdown()
    return 0


def evaluate(args) -> int:
    from .checkpoint.inference import bind_inference_weights
    from .checkpoint.store import latest_step
    from .metrics.ranking import auc, calibration, gauc
    from .models.dlrm import DLRM

    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = _dlrm_cfg(args.model_config)
    step = args.step if args.step is not None else latest_step(args.checkpoint_dir)
    if step is None:
        raise SystemExit(f"no checkpoint under {args.checkpoint_dir}")
    w = bind_inference_weights(args.checkpoint_dir, step)
    model = DLRM(cfg, args.batch, max_bag_size=args.max_bag, device=dev, seed=0)
    w.load_model(model.dense)
    w.load_sparse(model.emb)
    data = _batches(args, cfg, args.batch, 0, 1, dev)
    scores, labels, groups = [], [], []
    for _ in range(args.batches):
        b = next(data)
        model.set_batch(b.dense.to(dev), b.labels.to(dev), b.offsets.to(dev), b.values.to(dev), non_blocking=False)
        scores.append(model.predict()[:, 0].clone())
        labels.append(model.labels[:, 0].clone())
        if args.gauc_feature is not None:
            groups.append(group_ids(b.offsets, b.values, args.gauc_feature, args.batch).to(dev))
    model.check()
    s, y = torch.cat(scores), torch.cat(labels)
    w.verify()
    out = {"step": step, "samples": int(s.numel()), "auc": auc(s, y), "calibration": calibration(s, y)}
    if groups:
        g = torch.cat(groups)
        keep = g >= 0
        out["gauc"] = gauc(s[keep], y[keep], g[keep])
    print("[MetricsAggregator] " + " ".join(f"{k}={v:.6g}" if isinstance(v, float) else f"{k}={v}"
                                             for k, v in out.items()), flush=True)
    print(json.dumps(out), flush=True)
    return 0


def load_recipe(spec: str, batch_size: int):
    """``module:attr`` -> a recipe (an object with ``model_builder()``, ``ranking_task()`` and
    ``trainer()``, e.g. a ``recipes.ranking.BaseRankingRecipe``): an instance is used as is with its
    batch size replaced, a class or a factory is called with ``batch_size``.  The module is imported by
    name, so the framework's packages keep no import of the applications."""
    import dataclasses
    import importlib

    mod, sep, attr = spec.partition(":")
    if not sep or not mod or not attr:
        raise SystemExit(f"--recipe wants module:attr, got {spec!r}")
    obj = getattr(importlib.import_module(mod), attr)
    if not isinstance(obj, type) and hasattr(obj, "ranking_task"):
        recipe = dataclasses.replace(obj, batch_size=batch_size) if dataclasses.is_dataclass(obj) else obj
    else:
        try:
            recipe = obj(batch_size=batch_size)
        except TypeError as e:
            raise SystemExit(f"{spec} is not a recipe factory taking batch_size: {e}") from e
    missing = [m for m in ("model_builder", "ranking_task", "trainer") if not hasattr(recipe, m)]
    if missing:
        raise SystemExit(f"{spec} did not give a recipe ({type(recipe).__name__} lacks {', '.join(missing)})")
    return recipe


def recipe_batch(builder, n_labels: int, B: int, seed: int, device):
    """A synthetic batch of the recipe's tables: (dense, label ids, offsets, values) on ``device``."""
    from .data.synthetic import synthetic_ranking_batch

    vocabs = [t.num_embeddings for t in builder.sparse_tables()]
    return synthetic_ranking_batch(B, vocabs, int(builder.num_dense), int(builder.max_bag_size), seed=seed,
                                   device=device, n_labels=n_labels)


def recipe(args) -> int:
    """Train an application recipe with ``RankingModelTrainer`` (fused embedding collection, the
    recipe's module on the flat fused optimizer, one CUDA graph per micro-step position), write
    checkpoints, resume from the newest one, then report per-target AUC on held-out batches."""
    import torch.distributed as dist

    from .checkpoint.store import CheckpointManager, latest_step
    from .metrics.ranking import auc
    from .parallel.dist import init_distributed, shutdown

    info = init_distributed(timeout_s=300)
    rank, world = info.rank, max(info.world_size, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    rec = load_recipe(args.recipe, args.batch_per_gpu)
    task = rec.ranking_task()
    builder = rec.model_builder()
    n_labels = int(task.objective.target_labels.shape[1])
    tr = rec.trainer(rank=rank, world_size=world, device=dev, use_graph=not args.no_graph, seed=args.seed,
                     accumulation_steps=args.accumulation_steps)
    mgr = CheckpointManager(args.checkpoint_dir) if args.checkpoint_dir else None
    start = 0
    if args.resume and mgr is not None and latest_step(args.checkpoint_dir) is not None:
        start = tr.restore_checkpoint(mgr)
    B, saved = rec.batch_size, False
    t0 = time.perf_counter()
    for step in range(start + 1, start + args.steps + 1):
        # the batch stream is a function of (seed, rank, step), so a resumed run continues it
        res = tr.train_step(*recipe_batch(builder, n_labels, B, (args.seed + 1) * 1_000_003 + 7919 * step + rank,
                                          dev))
        if rank == 0 and args.log_every and (step % args.log_every == 0 or step == start + args.steps):
            print(f"[recipe {rec.name}] step {step} loss {res.loss:.6f}", flush=True)
        if mgr is not None and args.save_every and step % args.save_every == 0:
            tr.save_checkpoint(mgr, step, incremental=args.incremental and saved)
            saved = True
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    scores, labels = [], []
    for k in range(args.eval_batches):
        d, lab, offs, vals = recipe_batch(builder, n_labels, B, 10_000_019 + 104_729 * k + rank, dev)
        scores.append(tr.predict(d, offs, vals))
        labels.append(task.objective.per_target(lab)[0])
    tr.check()
    out = {"recipe": rec.name, "steps": args.steps, "last_step": start + args.steps, "wall_s": wall,
           "samples_per_s": args.steps * B * world / wall}
    if scores:
        s_all, y_all = torch.cat(scores), torch.cat(labels)
        if world > 1:
            gs = [torch.empty_like(s_all) for _ in range(world)]
            gy = [torch.empty_like(y_all) for _ in range(world)]
            dist.all_gather(gs, s_all)
            dist.all_gather(gy, y_all)
            s_all, y_all = torch.cat(gs), torch.cat(gy)
        out["eval_samples"] = int(s_all.shape[0])
        for t, name in enumerate(task.objective.targets):
            out[f"auc_{name}"] = auc(s_all[:, t], y_all[:, t])
    if rank == 0:
        print(json.dumps(out), flush=True)
    tr.close()
    shutdown()
    return 0


def group_ids(offsets: torch.Tensor, values: torch.Tensor, feature: int, batch: int) -> torch.Tensor:
    """Per sample: the first id of its bag of sparse ``feature`` (-1 for an empty bag)."""
    offs = offsets.long().cpu()
    vals = values.long().cpu()
    start = offs[feature * batch:(feature + 1) * batch]
    lens = offs[feature * batch + 1:(feature + 1) * batch + 1] - start
    first = vals[start.clamp(max=max(vals.numel() - 1, 0))] if vals.numel() else torch.zeros_like(start)
    return torch.where(lens > 0, first, torch.full_like(first, -1))


def main(argv=None) -> int:
    args = _parser().parse_args(argv)
    if args.cmd == "train":
        return train(args)
    if args.cmd == "recipe":
        return recipe(args)
    return evaluate(args)


if __name__ == "__main__":
    sys.exit(main())
