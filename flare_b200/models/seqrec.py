"""Sequential-recommendation transformer (B200 fused path + PyTorch reference).

Model: tokens of jagged user histories are packed (``data.synthetic.SeqBatch``);
token embedding = item (dim 256) + [4 side embeddings of dim 64]; ``L`` pre-LN
causal transformer layers (8 heads x 32, FFN 1024, ReLU) with jagged attention
inside each sequence; final LayerNorm; next-item sampled softmax against 512
uniformly drawn negatives shared by the whole step.

Fused path (``SeqRec``), per rank, one kernel per op on static buffers:
  embeddings: the sharded embedding collection looks up item + side bags (one
    bag per token, bag size 1) and the 512 negatives as extra rows, so input,
    positive-target and negative lookups of the tied item table share one
    deduplicated sparse update;
  dense: QKV / V^T / Q^T / output / FFN GEMMs on tcgen05 (the projection weights
    are FSDP-sharded over all ranks and gathered inside the first GEMM that
    reads them), jagged attention (``ops.attention``), LayerNorm and loss
    kernels (``csrc/seqrec.cu``); biases and LayerNorm parameters are
    replicated with the fused ZeRO-1 update.
``SeqRecTorch`` is the same model in PyTorch autograd (numerics oracle and the
library baseline).  The reference has no sequential model; this is one of the
benchmark configurations built on the framework's layers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .._native import native
from ..data.synthetic import SeqBatch
from ..ops.attention import DMODEL, HEAD_DIM, HEADS, AttentionBuffers, jagged_attention_backward, \
    jagged_attention_forward, jagged_attention_reference
from ..ops.dense import cast_pad_bf16, colsum_
from ..ops.dist_gemm import DistGemm, DistGemmContext
from ..ops.gemm import gemm
from ..parallel.symm import SymmetricHeap
from ..sparse.collection import ShardedEmbeddingBagCollection
from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from ..training.flat import DenseOptimizerConfig, DenseState, FlatParams
from ..training.fsdp import FsdpGroup, FsdpWeight


@dataclass
class SeqRecConfig:
    item_rows: int = 100_000_000
    side_rows: int = 100_000
    num_side: int = 4
    side_dim: int = 64
    layers: int = 4
    ffn: int = 1024
    negatives: int = 512
    max_len: int = 512
    ln_eps: float = 1e-5
    dense_optimizer: DenseOptimizerConfig = field(
        default_factory=lambda: DenseOptimizerConfig(kind="adamw", learning_rate=1e-3, weight_decay=0.01))
    sparse_optimizer: SparseOptimizerConfig = field(
        default_factory=lambda: SparseOptimizerConfig(kind="adam", learning_rate=1e-3))

    def __post_init__(self):
        if self.num_side * self.side_dim != DMODEL:
            raise ValueError("the side embeddings must concatenate to the model width (256)")

    def tables(self) -> list[SparseTableSpec]:
        opt = self.sparse_optimizer
        t = [SparseTableSpec("item", self.item_rows, DMODEL, optimizer=opt, init_scale=0.05)]
        t += [SparseTableSpec(f"side{i}", self.side_rows, self.side_dim, optimizer=opt, init_scale=0.05)
              for i in range(self.num_side)]
        return t

    def dense_flops_per_token(self, mean_len: float) -> float:
        """Forward + backward FLOPs per token (projections, FFN, attention, sampled softmax)."""
        d, f = DMODEL, self.ffn
        per_layer = 2 * d * 3 * d + 2 * d * d + 2 * 2 * d * f + 2 * 2 * mean_len / 2 * d
        return 3.0 * (self.layers * per_layer + 2 * d * self.negatives)


def seqrec_init_weights(cfg: SeqRecConfig, seed: int) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    out = {}
    for l in range(cfg.layers):
        out[f"l{l}.wqkv"] = torch.randn(3 * DMODEL, DMODEL, generator=g) * 0.02
        out[f"l{l}.wo"] = torch.randn(DMODEL, DMODEL, generator=g) * 0.02 / math.sqrt(2 * cfg.layers)
        out[f"l{l}.w1"] = torch.randn(cfg.ffn, DMODEL, generator=g) * 0.02
        out[f"l{l}.w2"] = torch.randn(DMODEL, cfg.ffn, generator=g) * 0.02 / math.sqrt(2 * cfg.layers)
    return out


class SeqRec:
    """Fused sequential model for one rank (data parallel + FSDP over all ranks)."""

    def __init__(self, cfg: SeqRecConfig, nseq: int, T_cap: int, *, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, heap: SymmetricHeap | None = None, seed: int = 0,
                 values_capacity: int | None = None):
        if T_cap % 128:
            raise ValueError("token capacity must be a multiple of 128")
        self.cfg, self.nseq, self.T = cfg, nseq, T_cap
        self.rank, self.world = rank, world_size
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        N = cfg.negatives
        self.B_emb = T_cap + N
        F = 1 + cfg.num_side
        cap = values_capacity or (T_cap * F + N)
        if heap is None:
            d, f, L = DMODEL, cfg.ffn, cfg.layers
            wts = L * (3 * d * d + d * d + 2 * d * f + 4 * 64 * world_size * f) * 6
            emb = 4 * (F * self.B_emb + 1) + 4 * cap + 2 * 2 * self.B_emb * 2 * DMODEL
            heap = SymmetricHeap(int(1.3 * (wts + emb)) + (128 << 20), rank=rank, world_size=world_size, device=dev)
        self.heap = heap
        ctx = DistGemmContext(heap)
        self.ctx = ctx
        init = seqrec_init_weights(cfg, seed)

        params = FlatParams()
        for l in range(cfg.layers):
            params.register(f"l{l}.ln1.g", (DMODEL,), "ones")
            params.register(f"l{l}.ln1.b", (DMODEL,), "zeros")
            params.register(f"l{l}.ln2.g", (DMODEL,), "ones")
            params.register(f"l{l}.ln2.b", (DMODEL,), "zeros")
            params.register(f"l{l}.b1", (cfg.ffn,), "zeros")
            params.register(f"l{l}.b2", (DMODEL,), "zeros")
        params.register("lnf.g", (DMODEL,), "ones")
        params.register("lnf.b", (DMODEL,), "zeros")
        self.params = params
        self.dense = DenseState(params, cfg.dense_optimizer, device=dev, rank=rank, world_size=world_size,
                                heap=heap, seed=seed)
        fg = FsdpGroup(ctx, list(range(world_size)))
        opt, sd = cfg.dense_optimizer, self.dense.step_dev
        self.W = []
        for l in range(cfg.layers):
            ws = {}
            for name in ("wqkv", "wo", "w1", "w2"):
                w0 = init[f"l{l}.{name}"]
                ws[name] = FsdpWeight(fg, f"l{l}.{name}", w0.shape[0], w0.shape[1], init_scale=0, seed=0, opt=opt,
                                      step_dev=sd, full_init=w0)
            self.W.append(ws)
        self.fsdp_weights = [w for ws in self.W for w in ws.values()]

        self.emb = ShardedEmbeddingBagCollection(
            cfg.tables(), self.B_emb, max_bag_size=1, rank=rank, world_size=world_size, device=dev, heap=heap,
            optimizer=cfg.sparse_optimizer, seed=seed, values_capacity=cap)

        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        T = T_cap
        self.seq_offsets = torch.zeros(nseq + 1, dtype=torch.int32, device=dev)
        self.target_row = torch.full((T,), -1, dtype=torch.int32, device=dev)
        self.num_valid = torch.ones(1, dtype=torch.int32, device=dev)
        self.x = [torch.zeros(T, DMODEL, **bf) for _ in range(cfg.layers + 1)]
        self.a = [torch.zeros(T, DMODEL, **bf) for _ in range(cfg.layers)]
        self.h = [torch.zeros(T, DMODEL, **bf) for _ in range(cfg.layers)]
        self.f = [torch.zeros(T, DMODEL, **bf) for _ in range(cfg.layers)]
        self.u = [torch.zeros(T, cfg.ffn, **bf) for _ in range(cfg.layers)]
        self.stats = [torch.zeros(4, T, **f32) for _ in range(cfg.layers)]  # ln1 mean/rstd, ln2 mean/rstd
        self.att = [AttentionBuffers(T, dev) for _ in range(cfg.layers)]
        self.y = torch.zeros(T, DMODEL, **bf)
        self.statf = torch.zeros(2, T, **f32)
        self.logits = torch.zeros(T, N, **f32)
        self.dneg = torch.zeros(T, N, **bf)
        self.dy = torch.zeros(T, DMODEL, **bf)
        self.dpos = torch.zeros(T, **f32)
        self.loss_sum = torch.zeros(1, **f32)
        self.g = [torch.zeros(T, DMODEL, **bf) for _ in range(2)]  # ping-pong residual-stream gradients
        self.du = torch.zeros(T, cfg.ffn, **bf)
        self.df = torch.zeros(T, DMODEL, **bf)
        self.dh = torch.zeros(T, DMODEL, **bf)
        self.da = torch.zeros(T, DMODEL, **bf)
        self._build()
        if world_size > 1:
            from ..parallel.dist import barrier

            torch.cuda.synchronize(dev)
            barrier()

    # ------------------------------------------------------------ build ops
    def _build(self) -> None:
        cfg, ctx, ds, C = self.cfg, self.ctx, self.dense, native()
        T, N, eps = self.T, cfg.negatives, cfg.ln_eps
        pooled = self.emb.pooled_output
        grad_in = self.emb.grad_input
        E_neg = pooled[T:T + N, :DMODEL]
        ops = [("emb.forward", lambda: self.emb.forward(training=True)),
               ("embed_combine", lambda: C.seq_embed_combine(pooled.data_ptr(), pooled.stride(0), T,
                                                             self.x[0].data_ptr(), DMODEL))]
        cv, gv = ds.compute_view, ds.grad_view

        def ln_fwd(x, g, b, y, stat):
            return lambda: C.seq_layernorm_fwd(x.data_ptr(), x.stride(0), T, cv(g).data_ptr(), cv(b).data_ptr(), eps,
                                               y.data_ptr(), y.stride(0), stat[0].data_ptr(), stat[1].data_ptr())

        def ln_bwd(dy, x, g, b, stat, resid, dx):
            return lambda: C.seq_layernorm_bwd(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), T,
                                               cv(g).data_ptr(), stat[0].data_ptr(), stat[1].data_ptr(),
                                               resid.data_ptr() if resid is not None else 0,
                                               resid.stride(0) if resid is not None else 0, dx.data_ptr(),
                                               dx.stride(0), gv(g).data_ptr(), gv(b).data_ptr())

        offs = self.seq_offsets
        for l in range(cfg.layers):
            w, A, st = self.W[l], self.att[l], self.stats[l]
            ops.append((f"l{l}.ln1", ln_fwd(self.x[l], f"l{l}.ln1.g", f"l{l}.ln1.b", self.a[l], st[0:2])))
            ops.append((f"l{l}.qkv", DistGemm(ctx, self.a[l], w["wqkv"].full, A.qkv, gb=w["wqkv"].w)))
            ops.append((f"l{l}.vt", DistGemm(ctx, w["wqkv"].full[2 * DMODEL:], self.a[l], A.vt)))
            ops.append((f"l{l}.qt", DistGemm(ctx, w["wqkv"].full[:DMODEL], self.a[l], A.qt)))
            ops.append((f"l{l}.attn", lambda A=A: jagged_attention_forward(A, offs, self.nseq, cfg.max_len)))
            ops.append((f"l{l}.wo", DistGemm(ctx, A.out, w["wo"].full, self.h[l], gb=w["wo"].w, epi="residual",
                                             aux1=self.x[l])))
            ops.append((f"l{l}.ln2", ln_fwd(self.h[l], f"l{l}.ln2.g", f"l{l}.ln2.b", self.f[l], st[2:4])))
            ops.append((f"l{l}.ffn1", DistGemm(ctx, self.f[l], w["w1"].full, self.u[l], gb=w["w1"].w,
                                               bias=cv(f"l{l}.b1"), relu=True)))
            ops.append((f"l{l}.ffn2", DistGemm(ctx, self.u[l], w["w2"].full, self.x[l + 1], gb=w["w2"].w,
                                               bias=cv(f"l{l}.b2"), epi="residual", aux1=self.h[l])))
        xL = self.x[cfg.layers]
        ops.append(("lnf", ln_fwd(xL, "lnf.g", "lnf.b", self.y, self.statf)))
        # ---- sampled softmax loss against the shared negatives
        ops.append(("neg_logits", DistGemm(ctx, self.y, E_neg, self.logits)))
        ops.append(("loss.zero", self.loss_sum.zero_))
        sm = dict(y=self.y.data_ptr(), ldy=DMODEL, emb=pooled.data_ptr(), ldemb=pooled.stride(0),
                  target_row=self.target_row.data_ptr(), logits=self.logits.data_ptr(), ldlog=N, T=T, N=N,
                  num_valid=self.num_valid.data_ptr(), dneg=self.dneg.data_ptr(), lddneg=N, dy=self.dy.data_ptr(),
                  lddy=DMODEL, dpos=self.dpos.data_ptr(), loss_sum=self.loss_sum.data_ptr())
        ops.append(("sampled_softmax", lambda: C.seq_sampled_softmax(sm)))
        ops.append(("dy_neg", DistGemm(ctx, self.dneg, E_neg, self.dy, b_t=True, epi="residual", aux1=self.dy)))
        # dE_neg = dneg^T y reduces over all T tokens into a [N, 256] tile: split-K into fp32, then bf16 rows
        self.dE = torch.zeros(N, DMODEL, dtype=torch.float32, device=self.device)
        ops.append(("dE_neg.zero", self.dE.zero_))
        ops.append(("dE_neg", lambda: gemm(self.dneg, self.y, a_t=True, b_t=True, out=self.dE, accumulate=True)))
        ops.append(("dE_neg.cast", lambda: cast_pad_bf16(self.dE, grad_in[T:T + N, :DMODEL])))
        g_cur = self.g[0]
        ops.append(("lnf.bwd", ln_bwd(self.dy, xL, "lnf.g", "lnf.b", self.statf, None, g_cur)))
        # ---- layers, backward
        for l in reversed(range(cfg.layers)):
            w, A, st = self.W[l], self.att[l], self.stats[l]
            g_next = self.g[(cfg.layers - l) % 2]
            ops.append((f"l{l}.db2", lambda g=g_cur, l=l: colsum_(g, gv(f"l{l}.b2"))))
            ops.append((f"l{l}.ffn2.dx", DistGemm(ctx, g_cur, w["w2"].full, self.du, b_t=True, mask=self.u[l],
                                                  colsum=gv(f"l{l}.b1"))))
            ops.append((f"l{l}.ffn2.dW", self._wgrad(g_cur, self.u[l], w["w2"].grad)))
            ops.append((f"l{l}.ffn1.dx", DistGemm(ctx, self.du, w["w1"].full, self.df, b_t=True)))
            ops.append((f"l{l}.ffn1.dW", self._wgrad(self.du, self.f[l], w["w1"].grad)))
            ops.append((f"l{l}.ln2.bwd", ln_bwd(self.df, self.h[l], f"l{l}.ln2.g", f"l{l}.ln2.b", st[2:4], g_cur,
                                                self.dh)))
            ops.append((f"l{l}.wo.dx", DistGemm(ctx, self.dh, w["wo"].full, A.dout, b_t=True)))
            ops.append((f"l{l}.wo.dxT", DistGemm(ctx, w["wo"].full, self.dh, A.dout_t, a_t=True)))
            ops.append((f"l{l}.wo.dW", self._wgrad(self.dh, A.out, w["wo"].grad)))
            ops.append((f"l{l}.attn.bwd", lambda A=A: jagged_attention_backward(A, offs, self.nseq, cfg.max_len)))
            ops.append((f"l{l}.qkv.dx", DistGemm(ctx, A.dqkv, w["wqkv"].full, self.da, b_t=True)))
            ops.append((f"l{l}.qkv.dW", self._wgrad(A.dqkv, self.a[l], w["wqkv"].grad)))
            ops.append((f"l{l}.ln1.bwd", ln_bwd(self.da, self.x[l], f"l{l}.ln1.g", f"l{l}.ln1.b", st[0:2], self.dh,
                                                g_next)))
            g_cur = g_next
        ops.append(("embed_grad", lambda g=g_cur: C.seq_embed_grad_split(
            g.data_ptr(), DMODEL, self.y.data_ptr(), DMODEL, self.dpos.data_ptr(), self.target_row.data_ptr(), T,
            grad_in.data_ptr(), grad_in.stride(0))))
        self.fb_ops = ops
        upd = [("emb.backward", self.emb.backward), ("dense.apply", self.dense.apply)]
        upd += [(f"fsdp.{w.name}", lambda w=w: w.apply(self.dense.step)) for w in self.fsdp_weights]
        self.update_ops = upd

    @staticmethod
    def _wgrad(dy, x, out):
        return lambda: gemm(dy, x, a_t=True, b_t=True, out=out, accumulate=True)

    # ------------------------------------------------------------------ data
    def set_batch(self, b: SeqBatch, non_blocking: bool = True) -> None:
        self.seq_offsets.copy_(b.seq_offsets, non_blocking=non_blocking)
        self.target_row.copy_(b.target_row, non_blocking=non_blocking)
        self.num_valid.copy_(b.num_valid, non_blocking=non_blocking)
        self.emb.set_input(b.emb_offsets, b.emb_values, non_blocking=non_blocking)

    # ------------------------------------------------------------------ step
    def forward_backward(self) -> torch.Tensor:
        for _, op in self.fb_ops:
            op()
        return self.loss_sum

    def train_step(self) -> torch.Tensor:
        for _, op in self.fb_ops:
            op()
        for _, op in self.update_ops:
            op()
        return self.loss_sum

    def profile_step(self) -> list[tuple[str, float]]:
        evs = []
        for name, op in self.fb_ops + self.update_ops:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append((name, e))
            op()
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        torch.cuda.synchronize()
        return [(n, e.elapsed_time(evs[i + 1][1] if i + 1 < len(evs) else end)) for i, (n, e) in enumerate(evs)]

    def check(self) -> None:
        self.emb.check()
        self.ctx.check("SeqRec GEMMs")
        for A in self.att:
            A.status.check("attention")
        if self.dense.status is not None:
            self.dense.status.check("dense optimizer")

    def logical_weights(self) -> dict[str, torch.Tensor]:
        out = {w.name: w.gather_master().cpu() for w in self.fsdp_weights}
        master = self.dense.gather_master().cpu()
        for name, e in self.params.entries.items():
            out[name] = master[e.offset:e.offset + e.numel].reshape(e.shape).clone()
        return out


# ---------------------------------------------------------------------------
# PyTorch reference
# ---------------------------------------------------------------------------
class SeqRecTorch(nn.Module):
    """The same model in PyTorch autograd on packed tokens (fp32 by default)."""

    def __init__(self, cfg: SeqRecConfig, *, seed: int = 0, device=None):
        super().__init__()
        self.cfg = cfg
        dk = {"device": device}
        self.item = nn.Embedding(cfg.item_rows, DMODEL, **dk)
        self.sides = nn.ModuleList(nn.Embedding(cfg.side_rows, cfg.side_dim, **dk) for _ in range(cfg.num_side))
        self.ln1 = nn.ModuleList(nn.LayerNorm(DMODEL, eps=cfg.ln_eps, **dk) for _ in range(cfg.layers))
        self.ln2 = nn.ModuleList(nn.LayerNorm(DMODEL, eps=cfg.ln_eps, **dk) for _ in range(cfg.layers))
        self.wqkv = nn.ModuleList(nn.Linear(DMODEL, 3 * DMODEL, bias=False, **dk) for _ in range(cfg.layers))
        self.wo = nn.ModuleList(nn.Linear(DMODEL, DMODEL, bias=False, **dk) for _ in range(cfg.layers))
        self.w1 = nn.ModuleList(nn.Linear(DMODEL, cfg.ffn, **dk) for _ in range(cfg.layers))
        self.w2 = nn.ModuleList(nn.Linear(cfg.ffn, DMODEL, **dk) for _ in range(cfg.layers))
        self.lnf = nn.LayerNorm(DMODEL, eps=cfg.ln_eps, **dk)
        with torch.no_grad():
            w = seqrec_init_weights(cfg, seed)
            for l in range(cfg.layers):
                for name, mod in (("wqkv", self.wqkv), ("wo", self.wo), ("w1", self.w1), ("w2", self.w2)):
                    mod[l].weight.copy_(w[f"l{l}.{name}"])
                self.w1[l].bias.zero_()
                self.w2[l].bias.zero_()

    @torch.no_grad()
    def load_logical(self, w: dict[str, torch.Tensor]) -> "SeqRecTorch":
        for l in range(self.cfg.layers):
            for name, mod in (("wqkv", self.wqkv), ("wo", self.wo), ("w1", self.w1), ("w2", self.w2)):
                mod[l].weight.copy_(w[f"l{l}.{name}"])
            self.w1[l].bias.copy_(w[f"l{l}.b1"])
            self.w2[l].bias.copy_(w[f"l{l}.b2"])
            self.ln1[l].weight.copy_(w[f"l{l}.ln1.g"])
            self.ln1[l].bias.copy_(w[f"l{l}.ln1.b"])
            self.ln2[l].weight.copy_(w[f"l{l}.ln2.g"])
            self.ln2[l].bias.copy_(w[f"l{l}.ln2.b"])
        self.lnf.weight.copy_(w["lnf.g"])
        self.lnf.bias.copy_(w["lnf.b"])
        return self

    def forward_from_pooled(self, pooled: torch.Tensor, b: SeqBatch, T: int) -> torch.Tensor:
        """Mean sampled-softmax loss from pooled embeddings [T + N, 512] (the fused kernels' input)."""
        cfg = self.cfg
        x = pooled[:T, :DMODEL] + pooled[:T, DMODEL:2 * DMODEL]
        offs = b.seq_offsets
        for l in range(cfg.layers):
            a = self.ln1[l](x)
            qkv = self.wqkv[l](a)
            att = jagged_attention_reference(qkv, offs.cpu())
            h = x + self.wo[l](att)
            x = h + self.w2[l](torch.relu(self.w1[l](self.ln2[l](h))))
        y = self.lnf(x)
        tgt = b.target_row.long()
        m = tgt >= 0
        e_pos = pooled[tgt.clamp(min=0), :DMODEL]
        pos = (y * e_pos).sum(-1, keepdim=True)
        neg = y @ pooled[T:T + cfg.negatives, :DMODEL].t()
        logits = torch.cat([pos, neg], 1)
        loss = torch.logsumexp(logits, 1) - pos[:, 0]
        return (loss * m).sum() / float(b.num_valid.item())


__all__ = ["SeqRec", "SeqRecConfig", "SeqRecTorch", "seqrec_init_weights"]
