"""Equivalence check of the fused DCN-v2 path against the PyTorch model (1 or more GPUs).

Every rank runs the fused forward/backward on its own batch (tensor parallel
over TP pairs with the all-gather / reduce-scatter inside the GEMMs, FSDP
weights gathered inside the GEMMs).  Every rank then rebuilds the logical
model (gathering shards), runs ``DCNTorch`` in fp32 on the concatenation of
all ranks' batches, and compares the loss and every gradient (relative
Frobenius error).  Then one optimizer step runs (FSDP reduce-scatter + AdamW
fused, ZeRO-1 for the replicated parameters) and every updated weight is
compared with the fp32 AdamW update of the gathered gradients (max error in
units of the learning rate).  Prints ``DCN_OK`` on success.

    python -m flare_b200.testing.dcn_check                       # 1 GPU
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m flare_b200.testing.dcn_check                          # TP = 2
"""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

from flare_b200.data.synthetic import DLRMSyntheticData
from flare_b200.models.dcn import DCN, DCNConfig, DCNTorch, dcn_benchmark_tables
from flare_b200.parallel.dist import init_distributed, shutdown
from flare_b200.testing.dist_dlrm_check import concat_batches
from flare_b200.training.flat import adam_reference

VOCABS = [300, 5000, 64, 2000]


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _all_reduce(t: torch.Tensor, world: int) -> torch.Tensor:
    t = t.clone().contiguous()
    if world > 1:
        dist.all_reduce(t)
    return t


def _all_gather(t: torch.Tensor, world: int) -> list[torch.Tensor]:
    t = t.contiguous()
    if world == 1:
        return [t]
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return parts


def run(m: int = 128, deep=(256, 256), rank_dim: int = 64, dim: int = 64, tol: float = 5e-2) -> int:
    if "RANK" in os.environ:
        info = init_distributed(timeout_s=120)
        rank, world = info.rank, info.world_size
    else:
        rank, world = 0, 1
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DCNConfig(tables=dcn_benchmark_tables(VOCABS, dim), cross_rank=rank_dim, deep=tuple(deep), tp=2)
    gens = [DLRMSyntheticData(m, VOCABS, max_bag=8, seed=7, rank=r, device=dev, pos_rate=0.3) for r in range(world)]
    batches = [g.next() for g in gens]
    model = DCN(cfg, m, max_bag_size=8, rank=rank, world_size=world, device=dev, seed=3)
    b = batches[rank]
    model.set_batch(b.dense, b.labels, b.offsets, b.values)
    loss_sum = model.forward_backward()
    torch.cuda.synchronize()
    model.check()
    tp = model.tp

    # ---- fused gradients of the logical model
    grads = {}
    for l in range(cfg.cross_layers):
        grads[f"cross{l}.V"] = _all_reduce(model.V[l].grad, world)
        grads[f"cross{l}.U"] = _all_reduce(model.U[l].grad, world)
    for i, w in enumerate(model.deepW):
        parts = _all_gather(w.grad, world)
        shards = [sum(parts[d * tp + t] for d in range(world // tp)) for t in range(tp)]
        grads[f"deep{i}.W"] = torch.cat(shards, 0 if model.col_parallel[i] else 1) if tp > 1 else shards[0]
    flat = _all_reduce(model.dense.grad, world)
    for name, e in model.params.entries.items():
        grads[name] = flat[e.offset:e.offset + e.numel].reshape(e.shape)
    hw = grads["head.w"]
    grads["head.w"] = torch.cat([hw[:model.W], hw[model.ldW:]])
    dpooled = torch.cat(_all_gather(model.emb.grad_input.float(), world))
    loss = float(_all_reduce(loss_sum, world).item()) / model.global_B

    # ---- reference on the global batch
    logical = model.logical_weights()
    tables = model.emb.export_pieces()
    if world > 1:
        allt = [None] * world
        dist.all_gather_object(allt, tables)
        for t in allt:
            tables.update(t)
    ref = DCNTorch(cfg).to(dev)
    ref.load_logical({k: v.to(torch.bfloat16).float() if v.dim() == 2 else v for k, v in logical.items()})
    with torch.no_grad():
        for t, w in enumerate(model.emb.assemble_tables(tables, model.emb.tables)):
            ref.embs[t].weight.copy_(w.to(dev))
    gb = concat_batches(batches, len(VOCABS))
    pooled = ref.pooled(gb.offsets, gb.values, gb.dense.shape[0]).detach().to(torch.bfloat16).float()
    pooled.requires_grad_(True)
    dense = gb.dense.to(torch.bfloat16).float()
    logits = ref.forward_from_pooled(pooled, dense)
    ref_loss = torch.nn.functional.binary_cross_entropy_with_logits(logits, gb.labels.reshape(-1))
    ref_loss.backward()
    ref_grads = {}
    for l in range(cfg.cross_layers):
        ref_grads[f"cross{l}.V"] = ref.V[l].weight.grad
        ref_grads[f"cross{l}.U"] = ref.U[l].weight.grad
        ref_grads[f"cross{l}.b"] = ref.U[l].bias.grad
    for i, lin in enumerate(ref.deep):
        ref_grads[f"deep{i}.W"] = lin.weight.grad
        ref_grads[f"deep{i}.b"] = lin.bias.grad
    ref_grads["head.w"] = ref.head.weight.grad.reshape(-1)
    ref_grads["head.b"] = ref.head.bias.grad

    ref_l = float(ref_loss.detach())
    errs = {"loss": abs(loss - ref_l) / abs(ref_l)}
    for k, g in ref_grads.items():
        errs[k] = _rel(grads[k], g)
    errs["pooled"] = _rel(dpooled[:, :cfg.emb_width], pooled.grad)
    # ---- optimizer step: fused reduce-scatter + AdamW (FSDP and ZeRO-1 shards) vs
    # the fp32 reference update applied to the gathered gradients
    op = cfg.dense_optimizer.kernel_params(1)
    model.emb.backward()
    model.dense.apply()
    for w in model.fsdp_weights:
        w.apply(model.dense.step)
    torch.cuda.synchronize()
    model.check()
    after = model.logical_weights()
    for k, w0 in logical.items():
        w = w0.clone().float()
        adam_reference(w, grads[k].float().cpu(), torch.zeros_like(w), torch.zeros_like(w), op)
        errs["step:" + k] = float((after[k] - w).abs().max()) / (op["lr"] + 1e-12)
    bad = {k: v for k, v in errs.items() if not v < tol}
    print(f"[rank{rank}] world={world} tp={tp} loss={loss:.6f} ref={ref_l:.6f} "
          + " ".join(f"{k}={v:.2e}" for k, v in errs.items()), flush=True)
    ok = not bad
    if world > 1:
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
        shutdown()
    if ok and rank == 0:
        print("DCN_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(run())
