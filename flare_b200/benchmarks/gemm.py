"""GEMM throughput: tcgen05 tile GEMM, persistent tcgen05 GEMM, cuBLAS (torch.matmul).

    python -m flare_b200.benchmarks.gemm [--shapes 8192x2048x6672,...] [--iters 20] [--graph] [--bn 64,128] [--pair]

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


def _time(fn, iters, graph: bool = False):
    """Mean ms per launch.  With ``graph`` the ``iters`` launches are captured in one CUDA graph and the
    replay is timed, so host launch overhead (which exceeds a small GEMM's device time) is excluded."""
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    g = None
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(iters):
                    fn(i)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if g is not None:
        g.replay()
    else:
        for i in range(iters):
            fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="8192x2048x6672,8192x4096x2048,4096x512x6672,4096x6672x512,8192x8192x8192")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--graph", action="store_true", help="time a CUDA graph of the launches (device time only)")
    ap.add_argument("--bn", default="", help="also run the tile kernel at these tile widths, e.g. 64,128,256")
    ap.add_argument("--no-persistent", action="store_true")
    ap.add_argument("--pair", action="store_true", help="also run CTA-pair (cta_group::2) tiles at widths 128 and 256")
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
        runs = {"tcgen05_tile": lambda i: gemm(As[i % copies], Bs[i % copies], out=Cs[i % copies])}
        for bn in (int(x) for x in args.bn.split(",") if x):
            runs[f"tcgen05_tile_bn{bn}"] = lambda i, bn=bn: gemm(As[i % copies], Bs[i % copies], out=Cs[i % copies],
                                                                 bn=bn)
        if args.pair:
            for bn in (128, 256):
                runs[f"tcgen05_pair_bn{bn}"] = lambda i, bn=bn: gemm(As[i % copies], Bs[i % copies],
                                                                     out=Cs[i % copies], bn=bn, pair=True)
        if not args.no_persistent:
            runs["tcgen05_persistent"] = lambda i: dg[i % copies]()
        runs["cublas"] = lambda i: torch.matmul(As[i % copies], Bs[i % copies].t(), out=Cs[i % copies])
        for name, fn in runs.items():
            ms = _time(fn, args.iters, graph=args.graph)
            print(json.dumps({"shape": shape, "kernel": name, "ms": round(ms, 4), "graph": args.graph,
                              "tflops": round(flops / ms / 1e9, 1)}), flush=True)
        ctx.check()


if __name__ == "__main__":
    main()
