"""Multi-GPU equivalence check for the fused DLRM path (run under torch.distributed.run).

Every rank trains the world-size-W model on its own batch; rank 0 also trains a
world-size-1 model on the concatenation of all ranks' batches.  After K steps
the sharded tables and the dense parameters must agree (fp32 tolerance).  This
exercises the in-kernel ids / pooled / gradient all-to-alls over NVLink peer
memory, the table/column-wise planner and the fused ZeRO-1 dense update;
``CHECK_ROW_SHARDS=N`` adds row-wise (modulo) pieces and their partial sums.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        -m flare_b200.testing.dist_dlrm_check
"""
from __future__ import annotations

import os
import sys
from dataclasses import replace

import torch
import torch.distributed as dist

from flare_b200.data.synthetic import DLRMSyntheticData, SparseBatch
from flare_b200.models.dlrm import DLRMConfig, dlrm_benchmark_tables
from flare_b200.parallel.dist import init_distributed, shutdown
from flare_b200.sparse.config import SparseOptimizerConfig
from flare_b200.training.trainer import DLRMTrainer

VOCABS = [300, 5000, 64, 20000, 1000, 7000, 150]


def concat_batches(batches: list[SparseBatch], F: int) -> SparseBatch:
    """Concatenate keyed-jagged batches along the sample axis (feature-major layout)."""
    B = [b.dense.shape[0] for b in batches]
    vals, offs = [], [0]
    for f in range(F):
        for b, n in zip(batches, B):
            o = b.offsets.long()
            seg = o[f * n:(f + 1) * n + 1]
            vals.append(b.values[seg[0]:seg[-1]])
            offs.extend((seg[1:] - seg[0] + offs[-1]).tolist())
    return SparseBatch(torch.cat([b.dense for b in batches]), torch.cat([b.labels for b in batches]),
                       torch.tensor(offs, dtype=torch.int32, device=batches[0].values.device), torch.cat(vals))


def export_tables(trainer: DLRMTrainer) -> dict:
    return trainer.model.emb.export_pieces()


def main(steps: int = 3, B: int = 128, row_shards: int = 1) -> int:
    """``row_shards > 1`` cuts tables 1 and 3 into that many row-wise (modulo) pieces."""
    info = init_distributed(timeout_s=120)
    rank, world = info.rank, info.world_size
    dev = torch.device("cuda", torch.cuda.current_device())
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    base = dlrm_benchmark_tables(VOCABS, 64, opt)
    tables = [replace(t, shards=row_shards) if i in (1, 3) else t for i, t in enumerate(base)]
    cfg = DLRMConfig(tables=tables, bottom=(128, 64), top=(128, 64), sparse_optimizer=opt)
    ref_cfg = replace(cfg, tables=base)
    gens = [DLRMSyntheticData(B, VOCABS, max_bag=10, seed=7, rank=r, device=dev, pos_rate=0.3) for r in range(world)]
    data = [[g.next() for _ in range(steps)] for g in gens]
    tr = DLRMTrainer(cfg, B, max_bag_size=10, rank=rank, world_size=world, device=dev, seed=11, use_graph=False)
    losses = [tr.train_step(data[rank][k]).loss for k in range(steps)]
    torch.cuda.synchronize()
    tr.check()
    tables = export_tables(tr)
    gathered = [None] * world
    dist.all_gather_object(gathered, tables)
    master = tr.model.dense.gather_master()
    ok = True
    if rank == 0:
        ref = DLRMTrainer(ref_cfg, B * world, max_bag_size=10, device=dev, seed=11, use_graph=False)
        for k in range(steps):
            ref.train_step(concat_batches([data[r][k] for r in range(world)], len(VOCABS)))
        torch.cuda.synchronize()
        merged = {k: v for part in gathered for k, v in part.items()}
        full = tr.model.emb.assemble_tables(merged, cfg.tables)
        want = ref.model.emb.assemble_tables(export_tables(ref), ref_cfg.tables)
        # After the first step the dense weights differ by fp32 summation order (per-rank partial sums
        # vs one batch), so the bf16 pooled gradients can differ by one bf16 ulp (2^-8 relative) and
        # each row-wise Adagrad step (about lr in size) by lr * 2^-8.  A row whose first gradient is
        # ~0 is the exception: Adagrad normalises it to a step of +-lr whatever its size, so a sign
        # flip moves it by 2 lr.  Bound the typical error tightly and allow such rows to be rare.
        tol = 2e-4 + 2.0 * opt.learning_rate * 2.0 ** -8 * (steps - 1)
        for t, w in enumerate(want):
            diff = (full[t] - w).abs()
            err = diff.max().item()
            frac = (diff > tol).float().mean().item()
            if (steps == 1 and err > tol) or frac > 2e-3 or err > 2.0 * opt.learning_rate * steps + 1e-6:
                print(f"table {t}: max abs diff {err}, fraction above {tol:.2e}: {frac:.2e}", file=sys.stderr)
                ok = False
        rd = ref.model.dense
        for name, e in tr.model.params.entries.items():
            got = master[e.offset:e.offset + e.numel]
            want = rd.master_view(name).reshape(-1)
            diff = (got - want).abs()
            # Adam normalises each element's step, so an element whose gradient
            # is ~0 can differ by up to lr per step when summation order flips
            # its sign; bound the maximum by steps*lr and the mean tightly.
            if diff.max().item() > 1.2e-3 * steps or diff.mean().item() > 2e-5:
                print(f"dense {name}: max {diff.max().item()} mean {diff.mean().item()}", file=sys.stderr)
                ok = False
        print(f"losses rank0 {losses}", file=sys.stderr)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    tr.close()
    shutdown()
    if rank == 0:
        print("DIST_OK" if flag.item() == 1 else "DIST_MISMATCH", flush=True)
    return 0 if flag.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main(int(os.environ.get("CHECK_STEPS", "3")), row_shards=int(os.environ.get("CHECK_ROW_SHARDS", "1"))))
