"""Host-DRAM-tier training throughput (tables larger than HBM).

    python -m flare_b200.benchmarks.tbscale --steps 10 --warmup 5
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m flare_b200.benchmarks.tbscale --gpus 8

Config: 8 tables x ``--rows-per-table`` rows x dim 128 fp32 kept in pinned host
memory (row-wise Adagrad state with them), an HBM cache of ``--cache-frac``
(10 %) of every table's rows; ids Zipf(1.05), bags U[1, 32], sum pooling; the
DLRM-style dense model (bottom 13-512-256-128, top 1024-1024-512-256-1, Adam);
16,384 samples per GPU (global 131,072 at 8 GPUs).  The full configuration is
8 x 250M rows (~1 TB); the host memory of the machine bounds ``--rows-per-table``
(tables are owned whole, so the host copy of a rank's tables must fit).
Synthetic seeded data, random-init weights; timing as in the other benchmarks.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

METRIC = "host-tier (TB-scale) train samples/sec (device-timed, max over ranks)"


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch-per-gpu", type=int, default=16384)
    p.add_argument("--rows-per-table", type=float, default=1.25e7)
    p.add_argument("--cache-frac", type=float, default=0.10)
    p.add_argument("--num-batches", type=int, default=8)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args(argv)


def log(msg):
    print(f"[tbscale rank{os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr,
          flush=True)


def main(argv=None):
    args = parse(argv)
    from flare_b200._native import native
    from flare_b200.data.synthetic import DLRMSyntheticData
    from flare_b200.models.dlrm import DLRMConfig
    from flare_b200.parallel.dist import barrier, init_distributed, max_over_ranks, shutdown
    from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
    from flare_b200.training.flat import DenseOptimizerConfig
    from flare_b200.training.trainer import DLRMTrainer
    from flare_b200.utils.clocks import ClockSampler

    info = init_distributed(timeout_s=600)
    rank, world = info.rank, max(info.world_size, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    B = args.batch_per_gpu
    rows = int(args.rows_per_table)
    cache = max(1, int(rows * args.cache_frac))
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.01)
    tables = [SparseTableSpec(f"t{i}", rows, 128, optimizer=opt, cache_rows=cache) for i in range(8)]
    cfg = DLRMConfig(tables=tables, sparse_optimizer=opt,
                     dense_optimizer=DenseOptimizerConfig(kind="adam", learning_rate=1e-3))
    gen = DLRMSyntheticData(B, [rows] * 8, max_bag=32, min_bag=1, seed=args.seed, rank=rank, device=dev)
    batches = [gen.next() for _ in range(args.num_batches)]
    max_nnz = int(max_over_ranks(max(b.values.numel() for b in batches)))
    log(f"world={world} building model: 8 x {rows} rows in host memory, {cache} cache rows per table")
    t0w = time.time()
    trainer = DLRMTrainer(cfg, B, max_bag_size=32, rank=rank, world_size=world, device=dev, seed=args.seed,
                          use_graph=not args.no_graph, values_capacity=max_nnz + 1024)
    model = trainer.model
    tier = model.emb.host_tier
    log(f"built in {time.time() - t0w:.0f}s: host {tier.host_bytes() / 1e9:.1f} GB on this rank")
    stream = torch.cuda.current_stream(dev)

    def device_step(i):
        b = batches[i % len(batches)]
        model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=True)
        trainer._run_step()
        trainer.steps += 1

    for i in range(max(args.warmup, 3)):
        device_step(i)
        torch.cuda.synchronize()
    trainer.check()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        device_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    trainer.check()
    st = tier.stats()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": B * world / (ms / 1e3), "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Zipf ids, random-init weights)", "impl": "flare",
            "config": {"model": "DLRM-style, 8 tables x dim 128 in pinned host memory + 10% HBM cache",
                       "rows_per_table": rows, "tables": 8, "cache_rows_per_table": cache,
                       "global_batch": B * world, "bag": "U[1,32]", "sparse_optimizer": "rowwise_adagrad",
                       "host_bytes_rank0": st["host_bytes"], "cuda_graph": not args.no_graph,
                       "l2": "inputs larger than L2 (tables in host memory; distinct batches cycled)"},
            "clocks": clk, "gpu_launches": (trainer.launches_per_step or 0) * args.steps,
            "gpu_launches_per_step": trainer.launches_per_step,
            "native_so": os.path.basename(native().__file__)}), flush=True)
    trainer.close()
    shutdown()


if __name__ == "__main__":
    main()
