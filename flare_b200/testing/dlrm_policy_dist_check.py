"""Multi-GPU checks of the fused DLRM's step policies (run under torch.distributed.run).

* Accumulation windows: every rank trains with ``accumulation_steps=2`` on
  micro-batches (a, b); a second model with twice the batch trains one
  step per window on the union of (a, b).  The window is one optimizer step
  on the sum / 2 of the micro-batch gradients, which is the union's
  gradient, so the two models stay equal (up to fp32 summation order).
* Pipelined staleness 2: every rank trains with ``sparse_policy="pipelined",
  staleness=2``; a synchronous model emulates it by looking up tables that
  miss the last two sparse updates (each rank swaps its own shards: the
  lookups of step t read every owner's tables as of step t - 2).

Prints ``POLICY_DIST_OK`` on rank 0 when both hold.  Run with NVLS off:

    NCCL_NVLS_ENABLE=0 python -m torch.distributed.run --nproc-per-node 2 \\
        --master-addr 127.0.0.1 -m flare_b200.testing.dlrm_policy_dist_check
"""
from __future__ import annotations

import sys

import torch
import torch.distributed as dist

from flare_b200.data.synthetic import DLRMSyntheticData, SparseBatch
from flare_b200.models.dlrm import DLRM, DLRMConfig, dlrm_benchmark_tables
from flare_b200.parallel.dist import barrier, init_distributed
from flare_b200.parallel.symm import SymmetricHeap
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig
from flare_b200.training.trainer import DLRMTrainer

VOCABS = [300, 5000, 64, 20000, 900]


def _cfg(kind: str = "sgd") -> DLRMConfig:
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05)
    return DLRMConfig(tables=dlrm_benchmark_tables(VOCABS, 64, opt), bottom=(64, 64), top=(128, 64),
                      sparse_optimizer=opt)


def _union(a: SparseBatch, b: SparseBatch, F: int, B: int) -> SparseBatch:
    offs, vals, base = [0], [], 0
    for f in range(F):
        for x in (a, b):
            seg = x.offsets[f * B:(f + 1) * B + 1].long()
            vals.append(x.values[seg[0]:seg[-1]])
            offs.extend((seg[1:] - seg[0] + base).tolist())
            base += int(seg[-1] - seg[0])
    dev = a.dense.device
    return SparseBatch(torch.cat([a.dense, b.dense]), torch.cat([a.labels, b.labels]),
                       torch.tensor(offs, dtype=torch.int32, device=dev), torch.cat(vals))


def _model(cfg, B, rank, world, dev, **kw) -> DLRM:
    heap = SymmetricHeap(ShardedEmbeddingBagCollection.exchange_bytes(
        cfg.tables, B, 8, pipelined=kw.get("sparse_policy") == "pipelined",
        pipeline_depth=max(1, kw.get("staleness") or 1), accumulation_steps=kw.get("accumulation_steps", 1))
        + (96 << 20), rank=rank, world_size=world, device=dev)
    m = DLRM(cfg, B, max_bag_size=8, rank=rank, world_size=world, device=dev, heap=heap, seed=7, **kw)
    torch.cuda.synchronize()
    barrier()
    return m


def check_windows(rank, world, dev) -> bool:
    cfg, B = _cfg("sgd"), 128  # SGD: a row's update is proportional to its gradient sum (no normalisation)
    win = _model(cfg, B, rank, world, dev, accumulation_steps=2)
    ref = _model(cfg, 2 * B, rank, world, dev, sparse_policy="sync")
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, seed=11, rank=rank, device=dev, pos_rate=0.3)
    for _ in range(4):
        a, b = data.next(), data.next()
        for x in (a, b):
            win.set_batch(x.dense, x.labels, x.offsets, x.values, non_blocking=False)
            win.train_step()
        u = _union(a, b, len(VOCABS), B)
        ref.set_batch(u.dense, u.labels, u.offsets, u.values, non_blocking=False)
        ref.train_step()
    torch.cuda.synchronize()
    win.check()
    ref.check()
    dw = (win.emb.weights - ref.emb.weights).abs().max().item()
    diff = (win.dense.master - ref.dense.master).abs()
    dm = diff.max().item()
    # Adam divides by the gradient's own magnitude: an element whose gradient nearly cancels can move
    # by up to the learning rate on summation-order rounding; almost every element must agree closely
    lr = cfg.dense_optimizer.learning_rate
    frac = (diff > 1e-4).float().mean().item()
    ok = dw < 1e-4 and frac < 1e-3 and dm <= 8 * lr and win.emb.step == ref.emb.step == 4 \
        and win.dense.step == ref.dense.step == 4
    print(f"[rank{rank}] windows: max|dtable|={dw:.2e} max|dmaster|={dm:.2e} (>1e-4: {frac:.2e}) "
          f"steps={win.emb.step},{ref.emb.step}", flush=True)
    return ok


def check_staleness2(rank, world, dev) -> bool:
    cfg, B, d = _cfg("sgd"), 128, 2
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, seed=13, rank=rank, device=dev, pos_rate=0.3)
    batches = [data.next() for _ in range(7)]
    tr = DLRMTrainer(cfg, B, max_bag_size=8, rank=rank, world_size=world, device=dev, seed=7, use_graph=True,
                     sparse_policy="pipelined", staleness=d)
    piped = [tr.train_step(x).loss for x in batches]
    tr.flush_pending_updates()
    torch.cuda.synchronize()
    tr.check()
    ref = _model(cfg, B, rank, world, dev, sparse_policy="sync")
    hist, emu = [ref.emb.weights.clone()], []
    for t, x in enumerate(batches):
        ref.set_batch(x.dense, x.labels, x.offsets, x.values, non_blocking=False)
        cur = ref.emb.weights.clone()
        ref.emb.weights.copy_(hist[max(t - d, 0)])
        barrier()  # every owner has swapped in its stale shards before any rank looks up
        loss = ref.forward_backward()
        torch.cuda.synchronize()
        barrier()
        ref.emb.weights.copy_(cur)
        torch.cuda.synchronize()
        barrier()
        ref.emb.backward()
        ref.dense.apply()
        emu.append(float(loss.item()) / B)
        hist.append(ref.emb.weights.clone())
    torch.cuda.synchronize()
    ref.check()
    dl = max(abs(a - b) for a, b in zip(piped, emu))
    dw = (tr.model.emb.weights - ref.emb.weights).abs().max().item()
    print(f"[rank{rank}] staleness 2: max|dloss|={dl:.2e} max|dtable|={dw:.2e}", flush=True)
    ok = dl < 2e-3 and dw < 1e-3
    tr.close()
    return ok


def main() -> int:
    info = init_distributed(timeout_s=120)
    rank, world = info.rank, info.world_size
    dev = torch.device("cuda", torch.cuda.current_device())
    ok = check_windows(rank, world, dev)
    ok = check_staleness2(rank, world, dev) and ok
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0 and int(flag) == 1:
        print("POLICY_DIST_OK", flush=True)
    dist.destroy_process_group()
    return 0 if int(flag) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
