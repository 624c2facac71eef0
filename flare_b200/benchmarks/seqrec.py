"""Sequential-recommendation transformer training throughput.

    python -m flare_b200.benchmarks.seqrec --steps 10 --warmup 3          # 1 GPU
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m flare_b200.benchmarks.seqrec --gpus 8
    ... --impl torch                                                    # PyTorch + cuBLAS baseline (eager)

Config: 512 user histories per GPU (global 4,096 at 8 GPUs), lengths
U[32, 512], items Zipf(1.1) over a table of 12.5M rows per GPU (100M at 8
GPUs, dim 256, column-wise sharded, sparse Adam), 4 side tables of 1e5 x 64;
4 causal layers, 8 heads, FFN 1024; sampled softmax with 512 shared uniform
negatives; AdamW on FSDP-sharded dense weights; bf16 compute.  Synthetic
seeded data, random-init weights.  Timing as in the other benchmarks (CUDA
events between barriers, max over ranks).  Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

METRIC = "seqrec train sequences/sec (device-timed, max over ranks)"


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["flare", "torch"], default="flare")
    p.add_argument("--nseq-per-gpu", type=int, default=512)
    p.add_argument("--item-rows-per-gpu", type=float, default=1.25e7)
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--num-batches", type=int, default=3)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--profile-ops", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args(argv)


def log(msg):
    print(f"[seqrec rank{os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr,
          flush=True)


def main(argv=None):
    args = parse(argv)
    from flare_b200.data.synthetic import SeqSyntheticData
    from flare_b200.models.seqrec import SeqRecConfig
    from flare_b200.parallel.dist import barrier, init_distributed, max_over_ranks, shutdown
    from flare_b200.utils.clocks import ClockSampler

    info = init_distributed(timeout_s=300)
    rank, world = info.rank, max(info.world_size, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    nseq = args.nseq_per_gpu
    item_rows = int(args.item_rows_per_gpu * (world if args.impl == "flare" else 1))
    cfg = SeqRecConfig(item_rows=item_rows, layers=args.layers)
    # capacity: the largest packed batch over the pre-generated steps (same on every rank)
    probe = [SeqSyntheticData(nseq, item_rows=item_rows, seed=args.seed, rank=r, world=world, T_cap=1 << 30)
             for r in range(world)]
    T_max = 0
    for pr in probe:
        for s in range(args.num_batches):
            T_max = max(T_max, int((((pr._lengths(pr.rank, s) + 7) // 8) * 8).sum()))
    T_cap = (T_max + 127) // 128 * 128
    data = SeqSyntheticData(nseq, item_rows=item_rows, seed=args.seed, rank=rank, world=world, T_cap=T_cap,
                            device=dev)
    batches = [data.next() for _ in range(args.num_batches)]
    tokens = sum(b.tokens for b in batches) / len(batches)
    flops = cfg.dense_flops_per_token(272.0) * tokens
    config = {"model": f"seq transformer: {cfg.layers} causal layers, 8 heads x 32, FFN {cfg.ffn}, jagged attention, "
                       f"sampled softmax with {cfg.negatives} shared negatives; item table {item_rows} x 256 "
                       "+ 4 side tables 1e5 x 64", "global_batch": nseq * world, "seq_len": "U[32,512]",
              "tokens_per_gpu_mean": tokens, "token_capacity": T_cap, "sparse_optimizer": "adam",
              "dense_optimizer": "adamw", "l2": "inputs larger than L2 (item table >> 126 MB; distinct batches)"}

    if args.impl == "torch":
        ms = run_torch(args, cfg, batches, T_cap, dev)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": nseq * world / (ms / 1e3), "unit": "sequences/s",
                              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                              "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
                              "impl": "torch", "config": dict(config, parallelism="single GPU eager")}), flush=True)
        shutdown()
        return

    from flare_b200._native import native
    from flare_b200.training.trainer import SeqRecTrainer

    cap = int(max_over_ranks(max(b.emb_values.numel() for b in batches)))
    log(f"world={world} T_cap={T_cap} building model")
    trainer = SeqRecTrainer(cfg, nseq, T_cap, rank=rank, world_size=world, device=dev, seed=args.seed,
                            use_graph=not args.no_graph, values_capacity=cap + 1024)
    model = trainer.model
    stream = torch.cuda.current_stream(dev)

    def device_step(i):
        model.set_batch(batches[i % len(batches)], non_blocking=True)
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
        log("per-op device times (eager, rank %d, total %.3f ms):\n" % (rank, total) +
            "\n".join(f"{n:24s} {ms:8.3f} ms {100 * ms / total:5.1f}%" for n, ms in prof))
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
        e2e_ms = max_over_ranks((time.perf_counter() - w0) * 1e3 / args.steps)
        bi = int(sum(t.numel() * t.element_size() for t in (host[0].seq_offsets, host[0].target_row,
                                                             host[0].emb_offsets, host[0].emb_values,
                                                             host[0].num_valid)))
        e2e = {"value": nseq * world / (e2e_ms / 1e3), "unit": "sequences/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4,
               "api": "flare_b200.training.trainer.SeqRecTrainer.train_step_async",
               "last_loss": last.loss if last else None}
    trainer.check()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": nseq * world / (ms / 1e3), "unit": "sequences/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Zipf ids, random-init weights)", "impl": "flare",
            "config": dict(config, parallelism=f"dp{world} + fsdp{world} dense, column-wise sharded item table",
                           cuda_graph=not args.no_graph),
            "tokens_per_sec": tokens * world / (ms / 1e3), "dense_tflops_per_gpu": flops / (ms / 1e3) / 1e12,
            "clocks": clk, "e2e": e2e, "gpu_launches": (trainer.launches_per_step or 0) * args.steps,
            "gpu_launches_per_step": trainer.launches_per_step,
            "native_so": os.path.basename(native().__file__)}), flush=True)
    trainer.close()
    shutdown()


def run_torch(args, cfg, batches, T_cap, dev) -> float:
    """PyTorch eager reference model (bf16 autocast, cuBLAS, per-sequence SDPA) on one GPU."""
    from flare_b200.models.seqrec import SeqRecTorch
    from flare_b200.ops.attention import DMODEL

    model = SeqRecTorch(cfg, device=dev)
    for e in [model.item] + list(model.sides):
        e.sparse = True
    dense = [p for n, p in model.named_parameters() if not (n.startswith("item") or n.startswith("sides"))]
    opt_d = torch.optim.AdamW(dense, lr=1e-3, weight_decay=0.01)
    opt_s = torch.optim.SGD(list(model.item.parameters()) + list(model.sides.parameters()), lr=0.01)
    F = 1 + cfg.num_side
    B = T_cap + cfg.negatives

    def step(i):
        b = batches[i % len(batches)]
        lens = (b.emb_offsets[1:] - b.emb_offsets[:-1]).view(F, B)
        starts = b.emb_offsets[:-1].view(F, B).long()
        ids = [torch.where(lens[f] > 0, b.emb_values[starts[f].clamp(max=b.emb_values.numel() - 1)].long(),
                           torch.zeros_like(starts[f])) for f in range(F)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            item = model.item(ids[0]) * (lens[0] > 0).unsqueeze(1)
            sides = torch.cat([model.sides[k](ids[k + 1]) * (lens[k + 1] > 0).unsqueeze(1)
                               for k in range(cfg.num_side)], 1)
            pooled = torch.cat([item, sides], 1)
            x = pooled[:T_cap, :DMODEL] + pooled[:T_cap, DMODEL:]
            offs = b.seq_offsets.tolist()
            for l in range(cfg.layers):
                a = model.ln1[l](x)
                qkv = model.wqkv[l](a)
                outs = []
                for s in range(len(offs) - 1):
                    q, k, v = qkv[offs[s]:offs[s + 1]].view(-1, 3, 8, 32).permute(1, 2, 0, 3)
                    outs.append(torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
                                .permute(1, 0, 2).reshape(-1, DMODEL))
                att = torch.zeros_like(x)
                att[:offs[-1]] = torch.cat(outs)
                h = x + model.wo[l](att)
                x = h + model.w2[l](torch.relu(model.w1[l](model.ln2[l](h))))
            y = model.lnf(x)
            tgt = b.target_row.long()
            pos = (y * pooled[tgt.clamp(min=0), :DMODEL]).sum(-1, keepdim=True)
            neg = y @ pooled[T_cap:, :DMODEL].t()
            loss = ((torch.logsumexp(torch.cat([pos, neg], 1).float(), 1) - pos[:, 0].float()) * (tgt >= 0)).sum() \
                / float(b.num_valid.item())
        opt_d.zero_grad(set_to_none=False)
        opt_s.zero_grad(set_to_none=True)
        loss.backward()
        opt_d.step()
        opt_s.step()

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / args.steps


if __name__ == "__main__":
    main()
