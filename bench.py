"""Headline benchmark: DLRM-style 26-table training throughput (samples/s).

    python bench.py --gpus N --steps K --warmup W            # this framework (fused sm_100a path)
    python bench.py --impl reference ...                      # the reference's own build (see below)
    python bench.py --impl torch ...                          # in-repo PyTorch/cuBLAS/NCCL baseline

For N > 1 launch one process per GPU with torch.distributed.run.  Per-GPU work
is fixed (weak scaling): each rank trains on ``--batch-per-gpu`` samples per
step (8192; global 65,536 at 8 GPUs) against 26 tables with log-uniform
vocabularies (1e3..4e7, 200M rows total, dim 128, fp32 storage) sharded over
the ranks' HBM.  Data is synthetic (seeded) and weights are random-init.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()`` on both sides, timed with CUDA events on the
training stream; the reported time is the max over ranks.  Each timed step
reads a different pre-generated batch, and the embedding tables (>100 GB per
node) are far larger than L2, so no L2 flush is needed.  SM clocks and throttle
reasons are sampled through NVML (read-only) during the timed region.  The e2e number
goes through ``DLRMTrainer.train_step_async`` with inputs in pinned host memory:
each step copies that step's inputs host->device and reads a loss back.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

METRIC = "train samples/sec (device-timed, max over ranks) at 1/2/4/8 B200; embed ms/step"
MODEL = "DLRM-style 26 tables + 13 dense (dim 128, ~200M rows, bottom 13-512-256-128, top 1024-1024-512-256-1)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["flare", "reference", "torch"], default="flare")
    p.add_argument("--batch-per-gpu", type=int, default=8192)
    p.add_argument("--total-rows", type=float, default=2e8)
    p.add_argument("--max-rows", type=float, default=4e7, help="largest table (smaller for small profiling cases)")
    p.add_argument("--max-bag", type=int, default=64)
    p.add_argument("--num-batches", type=int, default=16, help="distinct pre-generated batches cycled through")
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--profile-ops", action="store_true", help="also print a per-op eager breakdown (stderr)")
    p.add_argument("--plan", choices=["uniform", "cost", "cost-rw"], default="uniform",
                   help="table placement: by columns only; weighted by sampled per-table work; and also "
                        "splitting heavy tables into row-wise pieces")
    p.add_argument("--sparse-policy", choices=["sync", "pipelined"], default="sync",
                   help="pipelined: the sparse update of step t-1 overlaps step t's dense work (lookups one "
                        "step stale)")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def emit(obj):
    print(json.dumps(obj), flush=True)


_T0 = time.time()


def log(msg: str) -> None:
    """Progress line on stderr (rank-tagged)."""
    print(f"[bench rank{os.environ.get('RANK', '0')} +{time.time() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def reference_arm(args):
    """Run the unmodified reference through its own public API, if it can be imported."""
    ref_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    sys.path.insert(0, ref_dir)
    missing = []
    # the reference's training path (recipes/recsys/ranking) needs all of these
    for mod in ("flare", "flare.kernels", "jax", "flax", "fluxway", "sparse_embedding", "ray", "cupy"):
        try:
            __import__(mod)
        except Exception:  # noqa: BLE001
            missing.append(mod)
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if missing:
        emit({"impl": "reference", "unavailable": "reference installed offline with --no-deps into baseline/_ref "
              "(its deps are not in the wheelhouse), but its training stack cannot import: missing "
              + ", ".join(missing) + " (fluxway and sparse_embedding are not vendored; jax/ray/cupy not installed)"})
        return
    emit({"impl": "reference", "unavailable": "reference imports but its Ray/Fluxway cluster launch is not "
                                              "supported offline in this harness"})


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    from flare_b200.data.synthetic import DLRMSyntheticData, log_uniform_vocab_sizes
    from flare_b200.models.dlrm import DLRMConfig, dlrm_benchmark_tables
    from flare_b200.parallel.dist import barrier, init_distributed, max_over_ranks, shutdown
    from flare_b200.sparse.config import SparseOptimizerConfig
    from flare_b200.training.flat import DenseOptimizerConfig
    from flare_b200.utils.clocks import ClockSampler

    info = init_distributed(timeout_s=300)
    rank, world = info.rank, max(info.world_size, 1)
    if world != args.gpus and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", torch.cuda.current_device())
    B = args.batch_per_gpu
    vocabs = log_uniform_vocab_sizes(26, 1e3, args.max_rows, args.total_rows)
    sparse_opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.01)
    cfg = DLRMConfig(tables=dlrm_benchmark_tables(vocabs, 128, sparse_opt), sparse_optimizer=sparse_opt,
                     dense_optimizer=DenseOptimizerConfig(kind="adam", learning_rate=1e-3))

    log(f"world={world} building data")
    gens = DLRMSyntheticData(B, vocabs, max_bag=args.max_bag, seed=args.seed, rank=rank, device=dev)
    batches = [gens.next() for _ in range(args.num_batches)]
    # identical capacities on every rank (symmetric buffers)
    max_nnz = int(max_over_ranks(max(b.values.numel() for b in batches)))

    if args.impl == "torch":
        run_torch_baseline(args, cfg, batches, rank, world, dev)
        shutdown()
        return

    from flare_b200._native import native
    from flare_b200.training.trainer import DLRMTrainer

    costs = None
    if world > 1 and args.plan != "uniform":
        # per-table work of the global batch (lookups + the unique rows the backward updates), identical on
        # every rank (same seed): the planner balances it, splitting heavy tables into row-wise pieces
        from flare_b200.sparse.planner import estimate_table_costs

        costs = estimate_table_costs(vocabs, int(B * world * (args.max_bag + 1) / 2), 1.05, device=dev)
    trainer = DLRMTrainer(cfg, B, max_bag_size=args.max_bag, rank=rank, world_size=world, device=dev,
                          seed=args.seed, use_graph=not args.no_graph, values_capacity=max_nnz + 1024,
                          table_costs=costs, row_split=args.plan == "cost-rw", sparse_policy=args.sparse_policy)
    plan = trainer.model.emb.plan
    n_rw = len({p.table for p in plan.placements if p.row_shards > 1})
    model = trainer.model
    stream = torch.cuda.current_stream(dev)
    log(f"model built: {len(model.emb.shards)} local shards, {model.emb.memory_bytes() / 1e9:.1f} GB sparse state")

    def device_step(i):
        b = batches[i % len(batches)]
        model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=True)
        trainer._run_step()
        trainer.steps += 1

    for i in range(max(args.warmup, 3)):
        device_step(i)
        torch.cuda.synchronize()
        log(f"warmup step {i} done")
    trainer.check()
    launches_per_step = trainer.launches_per_step
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index).start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        device_step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    log("timed region done")
    ms = t0.elapsed_time(t1) / args.steps
    ms_max = max_over_ranks(ms)
    trainer.check()

    # embedding-only time (fused fwd + bwd kernels) on this rank, for "embed ms/step"
    trainer.flush_pending_updates()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(3):
        b = batches[i % len(batches)]
        model.emb.set_input(b.offsets, b.values)
        model.emb.forward()
        model.emb.backward()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    embed_ms = max_over_ranks(e0.elapsed_time(e1) / 3)
    emb_stats = model.emb.last_step_stats()

    log("embedding-only timing done")
    if args.profile_ops:
        for i in range(2):
            b = batches[i % len(batches)]
            model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=True)
            prof = model.profile_step()
        tot = sum(t for _, t in prof)
        log(f"{len(model.emb.shards)} shards; per-op (eager, ms): " + ", ".join(f"{n}={t:.3f}" for n, t in prof) + f", total={tot:.3f}")
    # e2e through the public API: inputs in pinned host memory, loss read back every step
    e2e = None
    if not args.no_e2e:
        host = [b.to("cpu").pin_memory() for b in batches]
        n_e2e = args.e2e_steps or args.steps
        for i in range(2):
            trainer.train_step_async(host[i % len(host)])
        first = trainer.flush()
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        h0 = torch.cuda.Event(enable_timing=True)
        h1 = torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for i in range(n_e2e):
            trainer.train_step_async(host[i % len(host)])
        last = trainer.flush()
        h1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        e2e_ms = max_over_ranks(max(h0.elapsed_time(h1), wall * 1000.0) / n_e2e)
        bi = int(sum(t.numel() * t.element_size() for t in (host[0].dense, host[0].labels, host[0].offsets,
                                                             host[0].values)))
        e2e = {"value": B * world / (e2e_ms / 1000.0), "unit": "samples/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4,
               "api": "flare_b200.training.trainer.DLRMTrainer.train_step_async",
               "first_loss": first.loss if first else None, "last_loss": last.loss if last else None,
               "steps_trained_before_last_loss": trainer.steps}
    trainer.check()

    samples_s = B * world / (ms_max / 1000.0)
    if rank == 0:
        emit({
            "metric": METRIC, "value": samples_s, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded Zipf ids, random-init weights)",
            "impl": "flare",
            "config": {"model": MODEL, "global_batch": B * world, "batch_per_gpu": B, "seq_len": None,
                       "parallelism": f"dp{world} dense (fused ZeRO-1) + table/column/row-wise sharded embeddings",
                       "sharding_plan": ("uniform" if costs is None else "cost-weighted (lookups + 2 x unique rows)")
                       + f", {n_rw} tables in row-wise pieces",
                       "embed_shards_rank0": len(model.emb.shards),
                       "sparse_policy": args.sparse_policy if args.sparse_policy == "sync" else
                       "pipelined (sparse update of step t-1 beside step t's dense work; lookups one step stale)",
                       "tables": 26, "total_rows": sum(vocabs), "embedding_dim": 128,
                       "embedding_storage": "fp32", "sparse_optimizer": "rowwise_adagrad",
                       "dense_optimizer": "adam", "l2": "inputs larger than L2 (tables > 100 GB, "
                       f"{args.num_batches} distinct batches cycled)", "cuda_graph": not args.no_graph},
            "embed_ms_per_step": embed_ms,
            "embed_stats_rank0": emb_stats,
            "clocks": clk,
            "e2e": e2e,
            "gpu_launches": (launches_per_step or 0) * args.steps,
            "gpu_launches_per_step": launches_per_step,
            "native_so": os.path.basename(native().__file__),
        })
    trainer.close()
    shutdown()


def run_torch_baseline(args, cfg, batches, rank, world, dev):
    """Plain PyTorch: nn.EmbeddingBag + nn.Linear + autocast bf16, DDP/NCCL for the dense grads."""
    import torch.distributed as dist

    from flare_b200.models.dlrm import DLRMTorch
    from flare_b200.parallel.dist import barrier, max_over_ranks

    model = DLRMTorch(cfg, dtype=torch.bfloat16).to(dev)
    dense_params = [p for n, p in model.named_parameters() if not n.startswith("embs.")]
    if world > 1:
        for p in dense_params:
            dist.broadcast(p.data, 0)
    opt_d = torch.optim.Adam(dense_params, lr=1e-3)
    # the same sparse optimizer as the fused path (row-wise Adagrad); plain PyTorch has no sharded
    # embedding, so at N > 1 every rank keeps whole tables and applies every rank's sparse gradients
    from flare_b200.models.dlrm import RowwiseAdagradTorch

    opt_s = RowwiseAdagradTorch([p for n, p in model.named_parameters() if n.startswith("embs.")], lr=0.01,
                                all_gather_grads=world > 1)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        b = batches[i % len(batches)]
        out = model(b.dense, b.offsets, b.values)
        loss = torch.nn.functional.binary_cross_entropy_with_logits(out, b.labels)
        opt_d.zero_grad(set_to_none=False)
        opt_s.zero_grad()
        loss.backward()
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1) for p in dense_params])
            dist.all_reduce(flat)
            flat /= world
            o = 0
            for p in dense_params:
                n = p.numel()
                p.grad.copy_(flat[o:o + n].view_as(p))
                o += n
        opt_d.step()
        opt_s.step()
        return loss

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    if rank == 0:
        emit({"metric": METRIC, "value": args.batch_per_gpu * world / (ms / 1000.0), "unit": "samples/s",
              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
              "data": "synthetic", "impl": "torch",
              "config": {"model": MODEL, "global_batch": args.batch_per_gpu * world,
                         "parallelism": f"dp{world} (NCCL all-reduce of dense gradients), replicated tables "
                                        "(every rank applies every rank's sparse gradients)",
                         "sparse_optimizer": "rowwise_adagrad (plain PyTorch on nn.EmbeddingBag sparse gradients)",
                         "dense_optimizer": "adam (torch.optim)"}})


if __name__ == "__main__":
    main()
