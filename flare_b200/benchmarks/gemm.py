"""GEMM throughput: tcgen05 tile GEMM, persistent tcgen05 GEMM, cuBLAS (torch.matmul).

    python -m flare_b200.benchmarks.gemm [--shapes 8192x2048x6672,...] [--iters 20]

Each shape is M x N x K with C = A @ B^T, bf16 in, bf16 out.  Timed with CUDA
events after warm-up; inputs are rotated over enough copies that the operands
of consecutive launches do not share L2 (126 MB).  Prints one JSON line per
shape and kernel with TFLOP/s.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops.dist_gemm import DistGemm, DistGemmContext
from ..ops.gemm import gemm


class _Heap:
    def __init__(self, device):
        self.rank, self.world_size, self.device = 0, 1, device

    def alloc(self, shape, dtype):
        from ..parallel.symm import SymBuffer

        t = torch.zeros(*shape, dtype=dtype, device=self.device)
        return SymBuffer(t, 0, [t.data_ptr()])


def _time(fn, iters):
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="8192x2048x6672,8192x4096x2048,4096x512x6672,4096x6672x512,8192x8192x8192")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    ctx = DistGemmContext(_Heap(dev))
    for shape in args.shapes.split(","):
        M, N, K = (int(x) for x in shape.split("x"))
        per = 2 * (M * K + N * K + M * N)
        copies = max(2, min(8, int(3 * 126e6 // per) + 1))
        As = [torch.randn(M, K, device=dev).to(torch.bfloat16) for _ in range(copies)]
        Bs = [torch.randn(N, K, device=dev).to(torch.bfloat16) for _ in range(copies)]
        Cs = [torch.empty(M, N, device=dev, dtype=torch.bfloat16) for _ in range(copies)]
        dg = [DistGemm(ctx, As[i], Bs[i], Cs[i]) for i in range(copies)]
        flops = 2.0 * M * N * K
        runs = {
            "tcgen05_tile": lambda i: gemm(As[i % copies], Bs[i % copies], out=Cs[i % copies]),
            "tcgen05_persistent": lambda i: dg[i % copies](),
            "cublas": lambda i: torch.matmul(As[i % copies], Bs[i % copies].t(), out=Cs[i % copies]),
        }
        for name, fn in runs.items():
            ms = _time(fn, args.iters)
            print(json.dumps({"shape": shape, "kernel": name, "ms": round(ms, 4),
                              "tflops": round(flops / ms / 1e9, 1)}), flush=True)
        ctx.check()


if __name__ == "__main__":
    main()
