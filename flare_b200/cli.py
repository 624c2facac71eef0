"""Command-line entry points: train and eval of the fused DLRM-family model.

    python -m flare_b200.cli train --model-config model.yaml --batch-per-gpu 8192 --steps 1000 \\
        --checkpoint-dir ckpt --save-every 500 [--data DIR_OF_PARQUET] [--resume]
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m flare_b200.cli train ...
    python -m flare_b200.cli eval --model-config model.yaml --checkpoint-dir ckpt [--step S] --batches 8

``train`` builds the model from a model-structure file (``{"model": "dlrm",
"tables": [...], ...}``, see ``config.loader.load_model_config``), feeds it
either synthetic batches of the table vocabularies or Parquet files
(``label``, ``d0..``, ``s0..`` list columns) through the prefetching loader,
logs AUC / calibration / loss / throughput windows (console + optional JSONL)
and writes FULL then INCREMENTAL checkpoints.  ``eval`` binds an immutable
checkpoint step as inference weights (verified against its recorded file
evidence), loads it into a one-GPU model and reports AUC / calibration on
held-out batches.  Reference behaviour: the ranking recipe's train and eval
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
    return evaluate(args)


if __name__ == "__main__":
    sys.exit(main())
