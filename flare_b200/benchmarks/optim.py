"""Dense optimizer kernels: fused reduce-scatter + Adam (FSDP / ZeRO-1 shard) vs flat Adam.

    python -m flare_b200.benchmarks.optim [--rows 2048 --cols 6672 --iters 20]

Single GPU (group of one): the fused kernel still runs its group barrier, so
this measures its memory-bound loop.  Bytes per element: gradient read +
zeroing write (8), master/m/v read + write (24), bf16 copy write (2) = 34.
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--cols", type=int, default=6672)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    from flare_b200._native import native
    from flare_b200.ops.dist_gemm import DistGemmContext
    from flare_b200.parallel.symm import SymmetricHeap
    from flare_b200.training.flat import DenseOptimizerConfig
    from flare_b200.training.fsdp import FsdpGroup, FsdpWeight

    dev = torch.device("cuda", 0)
    n = args.rows * args.cols
    heap = SymmetricHeap(n * 6 + (64 << 20), rank=0, world_size=1, device=dev)
    ctx = DistGemmContext(heap)
    fg = FsdpGroup(ctx, [0])
    step = torch.zeros(1, dtype=torch.int32, device=dev)
    opt = DenseOptimizerConfig(kind="adamw", learning_rate=1e-3, weight_decay=0.01)
    w = FsdpWeight(fg, "w", args.rows, args.cols, init_scale=0.02, seed=0, opt=opt, step_dev=step,
                   full_init=torch.randn(args.rows, args.cols) * 0.02)
    flat = {k: torch.zeros(n, device=dev) for k in ("master", "grad", "m", "v")}
    comp = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    op = opt.kernel_params(1)
    op["step_ptr"] = step.data_ptr()

    def fused():
        w.apply(1)

    def flat_adam():
        native().adam_flat(dict(master=flat["master"].data_ptr(), grad=flat["grad"].data_ptr(),
                                m=flat["m"].data_ptr(), v=flat["v"].data_ptr(), compute_copy=comp.data_ptr(), n=n,
                                grad_scale=1.0, zero_grad=1, opt=op))

    for name, fn in (("adam_dp_fused(fsdp, group 1)", fused), ("adam_flat", flat_adam)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        print(json.dumps({"kernel": name, "elements": n, "ms": round(ms, 4),
                          "gbs": round(34 * n / ms / 1e6, 1)}), flush=True)
    ctx.check()


if __name__ == "__main__":
    main()
