"""Equivalence check of the fused sequential model against ``SeqRecTorch`` (1 or more GPUs).

Every rank runs the fused forward/backward on its own packed batch; the
PyTorch model then runs on the same pooled embeddings (the fused lookup's
output) and the two are compared: loss, every dense gradient and the pooled
embedding gradient (item, sides, shared negatives).  Then one optimizer step
runs (FSDP reduce-scatter + AdamW, ZeRO-1 for the replicated parameters) and
the updated weights are compared with the fp32 AdamW update of the
gradients summed over ranks.  Prints ``SEQREC_OK``.

    python -m flare_b200.testing.seqrec_check
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 -m flare_b200.testing.seqrec_check
"""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

from flare_b200.data.synthetic import SeqSyntheticData
from flare_b200.models.seqrec import SeqRec, SeqRecConfig, SeqRecTorch
from flare_b200.parallel.dist import init_distributed, shutdown
from flare_b200.training.flat import adam_reference


def _rel(a, b) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _sum(t: torch.Tensor, world: int) -> torch.Tensor:
    t = t.clone().contiguous()
    if world > 1:
        dist.all_reduce(t)
    return t


def run(tol: float = 5e-2) -> int:
    if "RANK" in os.environ:
        info = init_distributed(timeout_s=120)
        rank, world = info.rank, info.world_size
    else:
        rank, world = 0, 1
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = SeqRecConfig(item_rows=5000, side_rows=300, layers=2, max_len=304)
    nseq, T_cap = 6, 6 * 304 + 128
    T_cap = (T_cap + 127) // 128 * 128
    data = SeqSyntheticData(nseq, item_rows=cfg.item_rows, side_rows=cfg.side_rows, min_len=5, max_len=300,
                            negatives=cfg.negatives, T_cap=T_cap, seed=5, rank=rank, world=world, device=dev)
    b = data.next()
    model = SeqRec(cfg, nseq, T_cap, rank=rank, world_size=world, device=dev, seed=2)
    model.set_batch(b)
    loss_sum = model.forward_backward()
    torch.cuda.synchronize()
    model.check()

    # ---- reference on the same pooled embeddings
    logical = model.logical_weights()
    ref = SeqRecTorch(cfg, device=dev)
    ref.load_logical({k: (v.to(torch.bfloat16).float() if v.dim() == 2 else v) for k, v in logical.items()})
    pooled = model.emb.pooled_output.detach().float().clone().requires_grad_(True)
    loss_ref = ref.forward_from_pooled(pooled, b, T_cap)
    loss_ref.backward()
    errs = {"loss": abs(float(loss_sum.item()) / float(b.num_valid.item()) - float(loss_ref.detach()))
            / abs(float(loss_ref.detach()))}
    fused_grads = {w.name: w.grad for w in model.fsdp_weights}
    g = model.dense.grad
    for name, e in model.params.entries.items():
        fused_grads[name] = g[e.offset:e.offset + e.numel].reshape(e.shape)
    ref_grads = {}
    for l in range(cfg.layers):
        ref_grads[f"l{l}.wqkv"] = ref.wqkv[l].weight.grad
        ref_grads[f"l{l}.wo"] = ref.wo[l].weight.grad
        ref_grads[f"l{l}.w1"] = ref.w1[l].weight.grad
        ref_grads[f"l{l}.w2"] = ref.w2[l].weight.grad
        ref_grads[f"l{l}.b1"] = ref.w1[l].bias.grad
        ref_grads[f"l{l}.b2"] = ref.w2[l].bias.grad
        ref_grads[f"l{l}.ln1.g"] = ref.ln1[l].weight.grad
        ref_grads[f"l{l}.ln1.b"] = ref.ln1[l].bias.grad
        ref_grads[f"l{l}.ln2.g"] = ref.ln2[l].weight.grad
        ref_grads[f"l{l}.ln2.b"] = ref.ln2[l].bias.grad
    ref_grads["lnf.g"] = ref.lnf.weight.grad
    ref_grads["lnf.b"] = ref.lnf.bias.grad
    for k, v in ref_grads.items():
        errs[k] = _rel(fused_grads[k], v)
    gin = model.emb.grad_input.float()
    rows = torch.cat([torch.nonzero(b.target_row >= 0).flatten() + 1,
                      torch.arange(T_cap, T_cap + cfg.negatives, device=dev)])
    errs["d_item"] = _rel(gin[rows, :256], pooled.grad[rows, :256])
    tok = torch.nonzero(b.target_row >= 0).flatten()
    errs["d_side"] = _rel(gin[tok, 256:], pooled.grad[tok, 256:])

    # ---- optimizer step vs fp32 AdamW on the summed gradients
    grads = {k: _sum(v.float(), world).cpu() for k, v in fused_grads.items()}
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
        adam_reference(w, grads[k], torch.zeros_like(w), torch.zeros_like(w), op)
        errs["step:" + k] = float((after[k] - w).abs().max()) / op["lr"]

    bad = {k: v for k, v in errs.items() if not v < tol}
    print(f"[rank{rank}] world={world} loss={float(loss_ref.detach()):.5f} bad={sorted(bad)} "
          + " ".join(f"{k}={v:.1e}" for k, v in errs.items()), flush=True)
    ok = not bad
    if world > 1:
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
        shutdown()
    if ok and rank == 0:
        print("SEQREC_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(run())
