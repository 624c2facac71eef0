"""DCN-v2 (tensor-parallel x FSDP) training throughput.

    python -m flare_b200.benchmarks.dcn --steps 10 --warmup 3                 # 1 GPU
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m flare_b200.benchmarks.dcn --gpus 8                                 # 2-way TP x 4-way FSDP
    ... --impl torch                                                          # PyTorch + cuBLAS + NCCL baseline

Config: 26 tables (log-uniform vocabularies, dim 256, fp32, row-wise Adam),
13 dense features, 3 low-rank cross layers (rank 512) over the 6,669-wide
input in parallel with a 4 x 4096 ReLU tower, AdamW, bf16 compute, 4,096
samples per GPU (global 32,768 at 8 GPUs).  Table rows scale with the GPU
count (200M rows at 8 GPUs) so every GPU holds the same sparse state (weak
scaling).  Synthetic seeded data, random-init weights.  Timing: warm-up, then
K steps between barriers + synchronize, CUDA events, max over ranks; the
tables are far larger than L2.  Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

METRIC = "DCN-v2 train samples/sec (device-timed, max over ranks)"


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["flare", "torch"], default="flare")
    p.add_argument("--batch-per-gpu", type=int, default=4096)
    p.add_argument("--rows-per-gpu", type=float, default=2.5e7)
    p.add_argument("--max-bag", type=int, default=64)
    p.add_argument("--num-batches", type=int, default=3)
    p.add_argument("--tp", type=int, default=2)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--profile-ops", action="store_true", help="print per-op device times of one eager step")
    return p.parse_args(argv)


def log(msg):
    print(f"[dcn rank{os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def main(argv=None):
    args = parse(argv)
    from flare_b200.data.synthetic import DLRMSyntheticData, log_uniform_vocab_sizes
    from flare_b200.models.dcn import DCNConfig, dcn_benchmark_tables
    from flare_b200.parallel.dist import barrier, init_distributed, max_over_ranks, shutdown
    from flare_b200.utils.clocks import ClockSampler

    info = init_distributed(timeout_s=300)
    rank, world = info.rank, max(info.world_size, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    B = args.batch_per_gpu
    # fused path: tables sharded, rows grow with the GPU count; torch baseline: replicated tables of one GPU's share
    rows = args.rows_per_gpu * (world if args.impl == "flare" else 1)
    vocabs = log_uniform_vocab_sizes(26, 1e3, 4e7, rows)
    cfg = DCNConfig(tables=dcn_benchmark_tables(vocabs, 256), tp=args.tp)
    gen = DLRMSyntheticData(B, vocabs, max_bag=args.max_bag, seed=args.seed, rank=rank, device=dev)
    batches = [gen.next() for _ in range(args.num_batches)]
    max_nnz = int(max_over_ranks(max(b.values.numel() for b in batches)))
    flops = cfg.dense_flops_per_sample() * B
    config = {"model": "DCN-v2: 26 tables x dim 256 + 13 dense (6,669 wide), 3 cross layers rank 512 "
                       "|| 4 x 4096 ReLU tower, BCE", "global_batch": B * world, "batch_per_gpu": B,
              "seq_len": None, "total_rows": sum(vocabs), "embedding_storage": "fp32",
              "sparse_optimizer": "rowwise_adam", "dense_optimizer": "adamw",
              "l2": "inputs larger than L2 (tables >> 126 MB; distinct batches cycled)"}

    if args.impl == "torch":
        ms = run_torch(args, cfg, batches, rank, world, dev)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": B * world / (ms / 1e3), "unit": "samples/s",
                              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                              "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
                              "impl": "torch", "config": dict(config, parallelism=f"dp{world} (NCCL all-reduce), "
                                                                                   "replicated tables")}),
                  flush=True)
        shutdown()
        return

    from flare_b200._native import native
    from flare_b200.training.trainer import DCNTrainer

    log(f"world={world} building model")
    trainer = DCNTrainer(cfg, B, max_bag_size=args.max_bag, rank=rank, world_size=world, device=dev,
                         seed=args.seed, use_graph=not args.no_graph, values_capacity=max_nnz + 1024)
    model = trainer.model
    stream = torch.cuda.current_stream(dev)
    log(f"model built: tp={model.tp} fsdp={world // model.tp}, sparse state "
        f"{model.emb.memory_bytes() / 1e9:.1f} GB")

    def device_step(i):
        b = batches[i % len(batches)]
        model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=True)
        trainer._run_step()
        trainer.steps += 1

    for i in range(max(args.warmup, 3)):
        device_step(i)
        torch.cuda.synchronize()
    trainer.check()
    log("warm-up done")
    if args.profile_ops:
        model.profile_step()
        prof = model.profile_step()
        total = sum(ms for _, ms in prof)
        lines = [f"{name:28s} {ms:8.3f} ms {100 * ms / total:5.1f}%" for name, ms in prof]
        log("per-op device times (eager, rank %d, total %.3f ms):\n" % (rank, total) + "\n".join(lines))
        trainer.steps += 2
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index).start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        device_step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    trainer.check()
    e2e = None
    if not args.no_e2e:
        host = [b.to("cpu").pin_memory() for b in batches]
        for i in range(2):
            trainer.train_step_async(host[i % len(host)])
        trainer.flush()
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for i in range(args.steps):
            trainer.train_step_async(host[i % len(host)])
        last = trainer.flush()
        wall = (time.perf_counter() - w0) * 1e3 / args.steps
        e2e_ms = max_over_ranks(wall)
        bi = int(sum(t.numel() * t.element_size() for t in (host[0].dense, host[0].labels, host[0].offsets,
                                                             host[0].values)))
        e2e = {"value": B * world / (e2e_ms / 1e3), "unit": "samples/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4,
               "api": "flare_b200.training.trainer.DCNTrainer.train_step_async",
               "last_loss": last.loss if last else None}
    trainer.check()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": B * world / (ms / 1e3), "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Zipf ids, random-init weights)", "impl": "flare",
            "config": dict(config, parallelism=f"tp{model.tp} x fsdp{world // model.tp} (fused AG/RS GEMMs) + "
                                               "table/column-wise sharded embeddings",
                           cuda_graph=not args.no_graph),
            "dense_tflops_per_gpu": flops / (ms / 1e3) / 1e12, "clocks": clk, "e2e": e2e,
            "gpu_launches": (trainer.launches_per_step or 0) * args.steps,
            "gpu_launches_per_step": trainer.launches_per_step,
            "native_so": os.path.basename(native().__file__)}), flush=True)
    trainer.close()
    shutdown()


def run_torch(args, cfg, batches, rank, world, dev) -> float:
    """PyTorch eager: EmbeddingBag tables (SGD), bf16 autocast, AdamW, NCCL all-reduce of dense grads."""
    import torch.distributed as dist

    from flare_b200.models.dcn import DCNTorch
    from flare_b200.parallel.dist import barrier, max_over_ranks

    model = DCNTorch(cfg, seed=args.seed, dtype=torch.bfloat16, device=dev, sparse_grad=True)
    dense = [p for n, p in model.named_parameters() if not n.startswith("embs.")]
    opt_d = torch.optim.AdamW(dense, lr=1e-3, weight_decay=0.01)
    opt_s = torch.optim.SGD([p for n, p in model.named_parameters() if n.startswith("embs.")], lr=0.01)

    def step(i):
        b = batches[i % len(batches)]
        out = model(b.dense, b.offsets, b.values)
        loss = torch.nn.functional.binary_cross_entropy_with_logits(out, b.labels.reshape(-1))
        opt_d.zero_grad(set_to_none=False)
        opt_s.zero_grad(set_to_none=True)
        loss.backward()
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1) for p in dense])
            dist.all_reduce(flat)
            flat /= world
            o = 0
            for p in dense:
                p.grad.copy_(flat[o:o + p.numel()].view_as(p))
                o += p.numel()
        opt_d.step()
        opt_s.step()

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    t0.record(stream)
    for i in range(args.steps):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(t0.elapsed_time(t1) / args.steps)


if __name__ == "__main__":
    main()
