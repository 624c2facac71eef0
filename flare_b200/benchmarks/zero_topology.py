"""ZeRO topology benchmark: global against node-local shard scope on one model.

    python -m torch.distributed.run --nproc-per-node 4 --master-addr 127.0.0.1 \\
        -m flare_b200.benchmarks.zero_topology --stage 2 --node-size 2 --steps 20

Both runs train the same MLP from the same seed on the same batches through
``TrainEngine``; the benchmark checks that they end with the same parameters
(node scope changes where shards live, not the maths) and reports, per
scope, the step time (max over ranks, wall clock around a barrier) and the
bytes each rank moves per optimizer step, split into the part that crosses
nodes and the part that stays inside one.  Global scope reduce-scatters and
all-gathers over every rank, so every collective spans nodes; node scope
all-reduces over every rank once and all-gathers inside the node.  Gloo on
CPU, NCCL when CUDA is available.  Reference behaviour:
tools/validation/benchmark_zero_topology.py:1-4 and its test
tests/training/test_zero_topology_benchmark.py:9-28.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch
import torch.distributed as dist
import torch.nn as nn

from ..training.contracts import TrainingExecutionPlan, ZeroStage
from ..training.engine import TrainEngine
from ..training.flat import DenseOptimizerConfig


def _model(width: int, depth: int, seed: int) -> nn.Module:
    torch.manual_seed(seed)
    layers: list[nn.Module] = []
    for _ in range(depth):
        layers += [nn.Linear(width, width), nn.ReLU()]
    layers.append(nn.Linear(width, 1))
    return nn.Sequential(*layers)


def ring_bytes(n: int, ranks: int, kind: str, elem: int = 4) -> float:
    """Bytes one rank sends in a ring collective over ``ranks`` ranks of an ``n``-element buffer."""
    if ranks <= 1:
        return 0.0
    per = n * elem * (ranks - 1) / ranks
    return 2 * per if kind == "all_reduce" else per


def step_bytes(scope: str, stage: int, n: int, world: int, node: int, wire: int) -> dict[str, float]:
    """Per-rank bytes of one optimizer step: (crossing nodes, inside a node).

    A collective over every rank counts as crossing nodes; an intra-node one as inside."""
    cross = inside = 0.0
    if stage == 0:
        cross += ring_bytes(n, world, "all_reduce", wire)
    elif scope == "global":
        cross += ring_bytes(n, world, "all_reduce" if stage == 1 else "reduce_scatter", wire)
        cross += ring_bytes(n, world, "all_gather")
    else:
        cross += ring_bytes(n, world, "all_reduce", wire)
        inside += ring_bytes(n, node, "all_gather")
    if stage == 3:  # parameters gathered again before the next window
        if scope == "global":
            cross += ring_bytes(n, world, "all_gather")
        else:
            inside += ring_bytes(n, node, "all_gather")
    return {"cross_node_bytes": cross, "intra_node_bytes": inside}


def run(rank: int, world: int, *, stage: int, node_size: int, steps: int, width: int = 256, depth: int = 3,
        batch: int = 64, micro: int = 1, device: torch.device | None = None) -> dict:
    dev = device or torch.device("cpu")
    out: dict = {"world": world, "node_size": node_size, "stage": stage, "scopes": {}}
    params = {}
    for scope in ("global", "node"):
        plan = TrainingExecutionPlan.sharded(ZeroStage(stage), micro_steps=micro, shard_scope=scope
                                             if stage > 0 else "global")
        eng = TrainEngine(_model(width, depth, 0).to(dev),
                          lambda o, y: nn.functional.binary_cross_entropy_with_logits(o, y), plan,
                          DenseOptimizerConfig(kind="adam", learning_rate=1e-3), device=dev, node_size=node_size)
        g = torch.Generator().manual_seed(1)
        data = [(torch.randn(batch * world, width, generator=g), (torch.rand(batch * world, 1, generator=g) < 0.5).float())
                for _ in range(4)]
        n_sl = slice(rank * batch, (rank + 1) * batch)
        dist.barrier()
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for s in range(steps):
            for m in range(micro):
                x, y = data[(s * micro + m) % len(data)]
                eng.micro_step_once(x[n_sl].to(dev), y[n_sl].to(dev))
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev if dev.type == "cuda" else "cpu")
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        params[scope] = eng.capture_checkpoint_state()["model_state"]
        out["scopes"][scope] = {"ms_per_step": 1000.0 * float(dt.item()) / steps, "shards": eng.shards,
                                **step_bytes(scope, stage, eng.padded, world, node_size if scope == "node" else world,
                                             eng.precision.gradient_transport_dtype.itemsize)}
    diff = max(float((params["global"][k] - params["node"][k]).abs().max()) for k in params["global"])
    out["max_param_diff_global_vs_node"] = diff
    return out


def main(argv=None) -> None:
    p = argparse.ArgumentParser(prog="zero_topology")
    p.add_argument("--stage", type=int, default=2, choices=[1, 2, 3])
    p.add_argument("--node-size", type=int, default=int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--width", type=int, default=256)
    p.add_argument("--depth", type=int, default=3)
    args = p.parse_args(argv)
    cuda = torch.cuda.is_available()
    dist.init_process_group("nccl" if cuda else "gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    res = run(rank, world, stage=args.stage, node_size=args.node_size, steps=args.steps, width=args.width,
              depth=args.depth, device=dev)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
