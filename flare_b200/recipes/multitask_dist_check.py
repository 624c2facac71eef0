"""2-GPU check of a user model on the fused path (run under torch.distributed.run).

Every rank trains the multitask PLE recipe (fused sharded embeddings, flat
fused optimizer: ZeRO-1 reduce-scatter + Adam + all-gather over NVLink peer
memory) on its own local batch; rank 0 also trains a one-GPU copy on the
concatenation of every rank's batch.  The global losses and the final dense
master weights and tables must agree (fp32 / bf16 tolerance).  The tables
train with SGD here: a row-wise Adagrad step normalises a row's gradient, so
a row whose summed gradient nearly cancels moves by up to the learning rate
on bf16 rounding differences alone (the per-sample gradients of a batch of B
and of 2B come from differently tiled GEMMs), which would hide a routing
error of the same size.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m flare_b200.recipes.multitask_dist_check
"""
from __future__ import annotations

import sys

import torch
import torch.distributed as dist

from flare_b200.parallel.dist import init_distributed
from flare_b200.recipes.multitask import MultitaskModelBuilder, MultitaskRankingRecipe, synthetic_multitask_batch
from flare_b200.sparse.config import SparseOptimizerConfig


def _concat(batches, F, B):
    dense = torch.cat([b[0] for b in batches])
    labels = torch.cat([b[1] for b in batches])
    vals, offs = [], [0]
    for f in range(F):
        for b in batches:
            o = b[2].long()
            seg = o[f * B:(f + 1) * B + 1]
            vals.append(b[3][seg[0]:seg[-1]])
            offs.extend((seg[1:] - seg[0] + offs[-1]).tolist())
    return dense, labels, torch.tensor(offs, dtype=torch.int32, device=dense.device), torch.cat(vals)


def main(steps: int = 4, B: int = 256) -> int:
    info = init_distributed(timeout_s=120)
    rank, world = info.rank, info.world_size
    dev = torch.device("cuda", torch.cuda.current_device())
    builder = MultitaskModelBuilder(sparse_optimizer=SparseOptimizerConfig(kind="sgd", learning_rate=0.05))
    recipe = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=B, builder=builder)
    data = [[synthetic_multitask_batch(B, builder.vocabs, builder.num_dense, builder.max_bag_size,
                                       seed=1000 * r + s, device=dev) for s in range(steps)] for r in range(world)]
    tr = recipe.trainer(rank=rank, world_size=world, device=dev, use_graph=True, seed=3)
    losses = []
    for s in range(steps):
        loss = torch.tensor([tr.train_step(*data[rank][s]).loss], device=dev)
        dist.all_reduce(loss)
        losses.append(float(loss))
    torch.cuda.synchronize()
    tr.check()
    master = tr.dense.state.gather_master()
    pieces = [None] * world
    dist.all_gather_object(pieces, tr.coll.export_pieces())
    ok = True
    if rank == 0:

        one = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=B * world, builder=builder)
        ref = one.trainer(device=dev, use_graph=True, seed=3)
        ref_losses = [ref.train_step(*_concat([data[r][s] for r in range(world)], len(builder.vocabs), B)).loss
                      for s in range(steps)]
        torch.cuda.synchronize()
        for s, (a, b) in enumerate(zip(losses, ref_losses)):
            if abs(a - b) > 2e-3 * max(1.0, abs(b)):
                print(f"[rank0] step {s} loss {a} vs {b}", flush=True)
                ok = False
        ref_master = ref.dense.state.gather_master()
        n = min(master.numel(), ref_master.numel())
        dm = (master[:n] - ref_master[:n]).abs().max().item()
        merged = {k: v for part in pieces for k, v in part.items()}
        full = tr.coll.assemble_tables(merged, tr.coll.tables)
        want = ref.coll.assemble_tables(ref.coll.export_pieces(), ref.coll.tables)
        dt = max((a - b).abs().max().item() for a, b in zip(full, want))
        print(f"[rank0] losses {losses} ref {ref_losses} max|dmaster|={dm:.2e} max|dtable|={dt:.2e}", flush=True)
        ok = ok and dm < 5e-3 and dt < 5e-3
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0 and int(flag) == 1:
        print("RECIPE_DIST_OK", flush=True)
    tr.close()
    dist.destroy_process_group()
    return 0 if int(flag) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
