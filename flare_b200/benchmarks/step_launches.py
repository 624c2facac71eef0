"""The kernels of replayed fused DLRM steps, inside an NVTX range for a launch-list capture.

    python -m flare_b200.benchmarks.step_launches --steps 3
    ncu --nvtx --nvtx-include "dlrm_step/" --metrics gpu__time_duration.sum --clock-control none \\
        --csv --log-file launches.csv python -m flare_b200.benchmarks.step_launches --steps 3

Builds a small DLRM-style model (26 tables of 20K rows, the benchmark's dense towers, batch 8192),
warms up past the CUDA-graph capture, then replays ``--steps`` training steps inside the NVTX range
``dlrm_step`` (inputs are copied in before the range), so the capture lists exactly what one
replayed step launches.
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=8192)
    args = ap.parse_args(argv)
    from ..data.synthetic import DLRMSyntheticData
    from ..models.dlrm import DLRMConfig, dlrm_benchmark_tables
    from ..training.trainer import DLRMTrainer

    dev = torch.device("cuda", 0)
    vocabs = [20_000] * 26
    cfg = DLRMConfig(tables=dlrm_benchmark_tables(vocabs, 128))
    tr = DLRMTrainer(cfg, args.batch, max_bag_size=64, device=dev, seed=0, use_graph=True)
    data = DLRMSyntheticData(args.batch, vocabs, max_bag=64, device=dev, seed=1)
    batch = data.next()
    for _ in range(4):
        tr.train_step(batch)
    m = tr.model
    torch.cuda.synchronize()
    for _ in range(args.steps):
        m.set_batch(batch.dense, batch.labels, batch.offsets, batch.values, non_blocking=True)
        torch.cuda.nvtx.range_push("dlrm_step")
        tr._run_step()
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    tr.check()
    print(json.dumps({"steps": args.steps, "launches_per_step_counted": tr.launches_per_step,
                      "graphs": len(tr.graphs)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
