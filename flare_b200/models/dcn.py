"""DCN-v2 ranking model on a tensor-parallel x FSDP mesh (B200 fused path + PyTorch reference).

Model (per sample): ``x0 = [pooled embeddings (26 x 256) | 13 dense]`` (6,669
wide); three low-rank cross layers ``x_{l+1} = x0 * (U_l (V_l x_l) + b_l) + x_l``
(rank 512) in parallel with a ReLU tower of four 4,096-wide layers; a logistic
head over ``[x_3, h_4]``; BCE loss.

Parallel layout on ``world = tp * fsdp`` GPUs (``parallel/mesh.py``):

* every rank trains its own ``B_local`` samples through the sharded embedding
  (tables sharded over all ranks, row-wise Adam);
* the deep tower is tensor parallel over each TP group with sequence
  (row) parallel activations: even layers are column-parallel and all-gather
  their input rows INSIDE the GEMM, odd layers are row-parallel and
  reduce-scatter their output rows INSIDE the GEMM (``ops/dist_gemm.py``);
  the backward mirrors it (the gradient of an all-gather is a
  reduce-scatter and vice versa);
* the cross layers run data parallel on the local rows: their FLOPs are
  small next to their activation bytes, so splitting them across the TP pair
  would move more data over NVLink than it saves in math;
* every large weight is FSDP-sharded (``training/fsdp.py``): the TP-sharded
  tower weights over the FSDP group, the cross weights over all ranks.  The
  parameter all-gather is fused into the first GEMM that reads the weight;
  the gradient reduce-scatter is fused with the AdamW update;
* biases and the head are small and replicated (ZeRO-1 fused update).

``DCN`` is the fused path (static buffers, one kernel per op, CUDA-graph
capturable).  ``DCNTorch`` is the same model in PyTorch autograd: the numerics
oracle and the library baseline.  The reference has no DCN model and no tensor
parallelism; its dense layers are Flax modules compiled by XLA
(src/flare/jax/layers/base.py:27) under its ZeRO engine
(src/flare/jax/training/engines/distributed.py:612-716).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .._native import native
from ..ops.dense import colsum_
from ..ops.dist_gemm import DistGemm, DistGemmContext, RowReduceScatter, ShardedRows
from ..ops.gemm import gemm
from ..parallel.mesh import DeviceMesh2D
from ..parallel.symm import SymmetricHeap
from ..sparse.collection import ShardedEmbeddingBagCollection
from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from ..training.flat import DenseOptimizerConfig, DenseState, FlatParams
from ..training.fsdp import FsdpGroup, FsdpWeight


ALIGN_SLACK = 4096  # per-buffer alignment slack in the symmetric heap estimate


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class DCNConfig:
    tables: list[SparseTableSpec]
    num_dense: int = 13
    cross_layers: int = 3
    cross_rank: int = 512
    deep: tuple[int, ...] = (4096, 4096, 4096, 4096)
    tp: int = 2
    dense_optimizer: DenseOptimizerConfig = field(
        default_factory=lambda: DenseOptimizerConfig(kind="adamw", learning_rate=1e-3, weight_decay=0.01))
    sparse_optimizer: SparseOptimizerConfig = field(
        default_factory=lambda: SparseOptimizerConfig(kind="rowwise_adam", learning_rate=1e-3))

    def __post_init__(self):
        dims = {t.embedding_dim for t in self.tables}
        if len(dims) != 1:
            raise ValueError("all tables share one embedding dim")
        if self.tp > 1 and len(self.deep) % 2:
            raise ValueError("a tensor-parallel tower needs column/row-parallel layer pairs")
        if any(d % (self.tp * 8) for d in self.deep):
            raise ValueError("tower widths must split evenly over the TP group")

    @property
    def embedding_dim(self) -> int:
        return self.tables[0].embedding_dim

    @property
    def emb_width(self) -> int:
        return len(self.tables) * self.embedding_dim

    @property
    def width(self) -> int:
        return self.emb_width + self.num_dense

    def dense_flops_per_sample(self) -> float:
        W, r = self.width, self.cross_rank
        f = self.cross_layers * 2 * (2 * W * r)
        dims = [W] + list(self.deep)
        f += sum(2 * a * b for a, b in zip(dims[:-1], dims[1:]))
        f += 2 * (W + self.deep[-1])
        return 3.0 * f


def dcn_benchmark_tables(vocab_sizes: list[int], dim: int = 256,
                         optimizer: SparseOptimizerConfig | None = None) -> list[SparseTableSpec]:
    opt = optimizer or SparseOptimizerConfig(kind="rowwise_adam", learning_rate=1e-3)
    return [SparseTableSpec(f"t{i}", int(v), dim, optimizer=opt) for i, v in enumerate(vocab_sizes)]


def dcn_init_weights(cfg: DCNConfig, seed: int) -> dict[str, torch.Tensor]:
    """Deterministic fp32 initial weights of the LOGICAL (unsharded) model, on the host."""
    g = torch.Generator().manual_seed(seed)
    W, r = cfg.width, cfg.cross_rank
    out = {}
    for l in range(cfg.cross_layers):
        out[f"cross{l}.V"] = torch.randn(r, W, generator=g) * (1.0 / W) ** 0.5
        out[f"cross{l}.U"] = torch.randn(W, r, generator=g) * (1.0 / r) ** 0.5
        out[f"cross{l}.b"] = torch.zeros(W)
    dims = [W] + list(cfg.deep)
    for i, (a, b) in enumerate(zip(dims[:-1], dims[1:])):
        out[f"deep{i}.W"] = torch.randn(b, a, generator=g) * (2.0 / a) ** 0.5
        out[f"deep{i}.b"] = torch.zeros(b)
    H = W + cfg.deep[-1]
    out["head.w"] = torch.randn(H, generator=g) * (1.0 / H) ** 0.5
    out["head.b"] = torch.zeros(1)
    return out


class DCN:
    """Fused DCN-v2 for one rank of the ``tp x fsdp`` mesh."""

    def __init__(self, cfg: DCNConfig, batch_size: int, *, max_bag_size: int, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, heap: SymmetricHeap | None = None, seed: int = 0,
                 values_capacity: int | None = None):
        self.cfg = cfg
        self.m = int(batch_size)
        self.rank, self.world = rank, world_size
        self.mesh = DeviceMesh2D.for_world(world_size, cfg.tp)
        tp = self.mesh.tp
        self.tp = tp
        self.tp_idx, self.dp_idx = self.mesh.coords(rank)
        self.global_B = self.m * world_size
        self.M = tp * self.m
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        if heap is None:
            heap = SymmetricHeap(self.heap_bytes(cfg, batch_size, world_size, max_bag_size, values_capacity),
                                 rank=rank, world_size=world_size, device=dev)
        self.heap = heap
        if self.m % 128 and tp > 1:
            raise ValueError("the local batch must be a multiple of 128 under tensor parallelism")
        ctx = DistGemmContext(heap)
        self.ctx = ctx
        W, r, L = cfg.width, cfg.cross_rank, cfg.cross_layers
        ldW = _round_up(W, 8)
        self.W, self.ldW = W, ldW
        E = cfg.emb_width
        self.E = E
        tp_group = self.mesh.tp_group(rank)
        fsdp_group = self.mesh.fsdp_group(rank)
        world_group = self.mesh.world_group()
        init = dcn_init_weights(cfg, seed)
        self._init = init

        # ---------------------------------------------------------- parameters
        params = FlatParams()
        for l in range(L):
            params.register(f"cross{l}.b", (W,), "zeros")
        for i, d in enumerate(cfg.deep):
            params.register(f"deep{i}.b", (d,), "zeros")
        H = ldW + cfg.deep[-1]
        self.H = H
        params.register("head.w", (H,), "zeros")
        params.register("head.b", (1,), "zeros")
        self.params = params
        self.dense = DenseState(params, cfg.dense_optimizer, device=dev, rank=rank, world_size=world_size,
                                heap=heap, seed=seed)
        hw = torch.zeros(H)
        hw[:W] = init["head.w"][:W]
        hw[ldW:] = init["head.w"][W:]
        self._load_replicated("head.w", hw)
        step_dev = self.dense.step_dev
        opt = cfg.dense_optimizer
        self.fsdp_tp = FsdpGroup(ctx, fsdp_group)
        self.fsdp_all = FsdpGroup(ctx, world_group) if fsdp_group != world_group else self.fsdp_tp
        self.V, self.U = [], []
        for l in range(L):
            self.V.append(FsdpWeight(self.fsdp_all, f"cross{l}.V", r, W, init_scale=0, seed=0, opt=opt,
                                     step_dev=step_dev, full_init=init[f"cross{l}.V"]))
            self.U.append(FsdpWeight(self.fsdp_all, f"cross{l}.U", W, r, init_scale=0, seed=0, opt=opt,
                                     step_dev=step_dev, full_init=init[f"cross{l}.U"]))
        dims = [W] + list(cfg.deep)
        self.deepW = []
        self.col_parallel = []
        for i, (a, b) in enumerate(zip(dims[:-1], dims[1:])):
            w = init[f"deep{i}.W"]
            colp = tp == 1 or i % 2 == 0
            if tp == 1:
                shard = w
            elif colp:  # output rows split over TP
                shard = w[self.tp_idx * (b // tp):(self.tp_idx + 1) * (b // tp)]
            else:       # input columns split over TP
                shard = w[:, self.tp_idx * (a // tp):(self.tp_idx + 1) * (a // tp)]
            self.col_parallel.append(colp)
            self.deepW.append(FsdpWeight(self.fsdp_tp, f"deep{i}.W", shard.shape[0], shard.shape[1], init_scale=0,
                                         seed=0, opt=opt, step_dev=step_dev, full_init=shard.contiguous()))
        self.fsdp_weights = self.V + self.U + self.deepW

        # ---------------------------------------------------------- embeddings
        self.emb = ShardedEmbeddingBagCollection(
            cfg.tables, self.m, max_bag_size=max_bag_size, rank=rank, world_size=world_size, device=dev, heap=heap,
            optimizer=cfg.sparse_optimizer, seed=seed, values_capacity=values_capacity)

        # ---------------------------------------------------------- activations
        bf = dict(dtype=torch.bfloat16, device=dev)
        m, M = self.m, self.M
        self.dense_in = torch.zeros(m, cfg.num_dense, dtype=torch.float32, device=dev)
        self.labels = torch.zeros(m, dtype=torch.float32, device=dev)
        self.x0 = ShardedRows(ctx, tp_group, m, W, ld=ldW)
        self.xs = [self.x0.local] + [torch.zeros(m, ldW, **bf) for _ in range(L - 1)]
        self.z = [torch.zeros(m, ldW, **bf) for _ in range(L)]
        self.t = [torch.zeros(m, r, **bf) for _ in range(L)]
        self.final_in = torch.zeros(m, H, **bf)
        nd = len(cfg.deep)
        self.h = []        # layer outputs: col-parallel [M, d/tp] tensors, row-parallel ShardedRows (local rows)
        self.rs = RowReduceScatter(ctx, tp_group, m, max(max(cfg.deep), W)) if tp > 1 else None
        for i, d in enumerate(cfg.deep):
            if self.col_parallel[i] and tp > 1:
                self.h.append(torch.zeros(M, d // tp, **bf))
            elif i == nd - 1:
                self.h.append(None)  # written into final_in
            elif tp > 1:
                self.h.append(ShardedRows(ctx, tp_group, m, d))
            else:
                self.h.append(torch.zeros(m, d, **bf))
        self.logits = torch.zeros(m, dtype=torch.float32, device=dev)
        self.dl = torch.zeros(m, dtype=torch.float32, device=dev)
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        # backward buffers
        self.dfin = ShardedRows(ctx, tp_group, m, H, ld=H)
        self.dz = torch.zeros(m, ldW, **bf)
        self.dt = torch.zeros(m, r, **bf)
        self.g = [torch.zeros(m, ldW, **bf) for _ in range(L)]  # g[l] = d x_l (l >= 1)
        self.dx0 = torch.zeros(m, ldW, dtype=torch.float32, device=dev)
        self.dpre = []
        for i, d in enumerate(cfg.deep):
            if self.col_parallel[i] and tp > 1:
                self.dpre.append(torch.zeros(M, d // tp, **bf))
            elif i == nd - 1:
                self.dpre.append(self.dfin.column_view(ldW, d) if tp > 1 else None)
            elif tp > 1:
                self.dpre.append(ShardedRows(ctx, tp_group, m, d))
            else:
                self.dpre.append(torch.zeros(m, d, **bf))
        self._build_calls()
        self._build_ops()
        if world_size > 1:
            # every rank's flags and buffers are initialised before any peer signals into them
            from ..parallel.dist import barrier

            torch.cuda.synchronize(dev)
            barrier()

    # ------------------------------------------------------------------ setup
    @staticmethod
    def heap_bytes(cfg: DCNConfig, batch_size: int, world_size: int, max_bag_size: int,
                   values_capacity: int | None = None) -> int:
        """Symmetric memory one rank needs: gathered activations, reduce-scatter slots, FSDP weights + grads,
        replicated dense state and the embedding exchange buffers."""
        tp = min(cfg.tp, world_size)
        W = _round_up(cfg.width, 8)
        m, M = batch_size, tp * batch_size
        H = W + cfg.deep[-1]
        acts = 2 * M * (W + H) + 2 * 2 * sum(M * d for d in cfg.deep)
        rs = 2 * tp * m * _round_up(max(max(cfg.deep), W), 8) + 4 * tp * (m // 128 + 1) * 64 * 4
        dims = [cfg.width] + list(cfg.deep)
        elems = 0
        for _ in range(cfg.cross_layers):
            elems += (cfg.cross_rank + 64 * world_size) * W + (cfg.width + 64 * world_size) * cfg.cross_rank
        for a, b in zip(dims[:-1], dims[1:]):
            elems += (b + 64 * world_size) * _round_up(a, 8)
        wts = 6 * elems  # bf16 compute copy + fp32 gradient
        small = 6 * (cfg.cross_layers * W + sum(cfg.deep) + H + 64 * 64) * 2
        emb = ShardedEmbeddingBagCollection.exchange_bytes(cfg.tables, batch_size, max_bag_size, values_capacity)
        return int(acts + rs + wts + small + emb) + 256 * ALIGN_SLACK + (64 << 20)

    def _load_replicated(self, name: str, value: torch.Tensor) -> None:
        e = self.params.entries[name]
        ds = self.dense
        full = value.reshape(-1).to(ds.device, torch.float32)
        lo, hi = e.offset, e.offset + e.numel
        a, b = max(lo, ds.lo), min(hi, ds.hi)
        if a < b:
            ds.master[a - ds.lo:b - ds.lo] = full[a - lo:b - lo]
        ds.compute[lo:hi] = full.to(ds.compute.dtype)

    def _build_calls(self) -> None:
        cfg, ctx = self.cfg, self.ctx
        W, ldW, L, tp = self.W, self.ldW, cfg.cross_layers, self.tp
        ds = self.dense
        nd = len(cfg.deep)
        self.fwd_calls, self.bwd_cross, self.bwd_deep = [], [], []
        # cross forward (local rows; weights FSDP-gathered inside the GEMM)
        for l in range(L):
            xl = self.xs[l][:, :W]
            self.fwd_calls.append((f"fwd.cross{l}.V", DistGemm(ctx, xl, self.V[l].full, self.t[l], gb=self.V[l].w)))
            out = self.final_in[:, :W] if l == L - 1 else self.xs[l + 1][:, :W]
            self.fwd_calls.append((f"fwd.cross{l}.U", DistGemm(ctx, self.t[l], self.U[l].full, out, gb=self.U[l].w,
                                                                bias=ds.compute_view(f"cross{l}.b"), epi="cross",
                                                                aux0=self.x0.local[:, :W], aux1=self.xs[l][:, :W],
                                                                zout=self.z[l][:, :W])))
        # deep forward
        a_in, a_sr = self.x0.full[:, :W], self.x0
        for i, d in enumerate(cfg.deep):
            w = self.deepW[i]
            bias = ds.compute_view(f"deep{i}.b")
            if self.col_parallel[i] and tp > 1:
                bsl = bias[self.tp_idx * (d // tp):(self.tp_idx + 1) * (d // tp)]
                self.fwd_calls.append((f"fwd.deep{i}.ag_gemm", DistGemm(ctx, a_in, w.full, self.h[i], ga=a_sr, gb=w.w,
                                                                        bias=bsl, relu=True)))
                a_in, a_sr = self.h[i], None
            else:
                if i == nd - 1:
                    out = self.final_in[:, ldW:]
                elif tp > 1:
                    out = self.h[i].local
                else:
                    out = self.h[i]
                self.fwd_calls.append((f"fwd.deep{i}.gemm_rs", DistGemm(ctx, a_in, w.full, out, gb=w.w, rs=self.rs,
                                                                        bias=bias, relu=True)))
                if i < nd - 1:
                    a_in = self.h[i].full[:, :d] if tp > 1 else self.h[i]
                    a_sr = self.h[i] if tp > 1 else None
        # cross backward: g_L = dfin[:, :W]
        for l in reversed(range(L)):
            g_next = self.dfin.local[:, :ldW] if l == L - 1 else self.g[l + 1]
            calls = []
            calls.append(("elem", l, g_next))
            calls.append((f"bwd.cross{l}.dt", DistGemm(ctx, self.dz[:, :W], self.U[l].full, self.dt, b_t=True)))
            if l > 0:
                calls.append((f"bwd.cross{l}.dx", DistGemm(ctx, self.dt, self.V[l].full, self.g[l][:, :W], b_t=True,
                                                           epi="residual", aux1=g_next[:, :W])))
            else:
                calls.append((f"bwd.cross{l}.dx", DistGemm(ctx, self.dt, self.V[l].full, self.dx0[:, :W], b_t=True,
                                                           epi="residual", aux1=g_next[:, :W], accumulate=True)))
            calls.append(("wgrad", f"bwd.cross{l}.dU", self.dz[:, :W], self.t[l], self.U[l].grad))
            calls.append(("wgrad", f"bwd.cross{l}.dV", self.dt, self.xs[l][:, :W], self.V[l].grad))
            self.bwd_cross.append(calls)
        # deep backward.  deep{i}.b gets colsum(dpre_i): from the head's output for
        # the last layer, otherwise from the epilogue of the GEMM producing dpre_i.
        dims = [W] + list(cfg.deep)
        for i in reversed(range(nd)):
            w = self.deepW[i]
            d_in = dims[i]
            prev_bias = ds.grad_view(f"deep{i - 1}.b") if i > 0 else None
            if self.col_parallel[i] and tp > 1:
                # column-parallel layer i: input rows gathered, output dpre[i] [M, d/tp]
                a_full = self.x0.full[:, :W] if i == 0 else self.h[i - 1].full[:, :d_in]
                if i == 0:
                    self.bwd_deep.append((f"bwd.deep{i}.dx_rs", DistGemm(ctx, self.dpre[i], w.full, self.dx0[:, :W],
                                                                         b_t=True, rs=self.rs, accumulate=True)))
                else:  # input came from a row-parallel layer: full-width local rows after the reduce-scatter
                    self.bwd_deep.append((f"bwd.deep{i}.dx_rs", DistGemm(ctx, self.dpre[i], w.full,
                                                                         self.dpre[i - 1].local, b_t=True, rs=self.rs,
                                                                         mask=self.h[i - 1].local, colsum=prev_bias)))
                self.bwd_deep.append(("wgrad", f"bwd.deep{i}.dW", self.dpre[i], a_full, w.grad))
                continue
            # row-parallel layer i (or any layer when tp == 1)
            last = i == nd - 1
            if tp > 1:
                dsr = self.dpre[i]
                d_full = dsr.full if last else dsr.full[:, :cfg.deep[i]]
                d_local = dsr.local
            else:
                dsr = None
                d_full = d_local = self.dfin.local[:, ldW:] if last else self.dpre[i]
            if last:
                self.bwd_deep.append(("colsum", f"bwd.deep{i}.db", d_local, ds.grad_view(f"deep{i}.b")))
            if i == 0:
                self.bwd_deep.append((f"bwd.deep{i}.ag_dx", DistGemm(ctx, d_full, w.full, self.dx0[:, :W], b_t=True,
                                                                     ga=dsr, accumulate=True)))
                self.bwd_deep.append(("wgrad", f"bwd.deep{i}.dW", d_full, self.x0.full[:, :W], w.grad))
                continue
            h_prev = self.h[i - 1]
            if tp > 1:  # previous layer is column-parallel: this rank's slice of its bias
                sl = dims[i] // tp
                prev_bias = prev_bias[self.tp_idx * sl:(self.tp_idx + 1) * sl]
            self.bwd_deep.append((f"bwd.deep{i}.ag_dx", DistGemm(ctx, d_full, w.full, self.dpre[i - 1], b_t=True,
                                                                 ga=dsr, mask=h_prev, colsum=prev_bias)))
            self.bwd_deep.append(("wgrad", f"bwd.deep{i}.dW", d_full, h_prev, w.grad))

    # ------------------------------------------------------------------ data
    def set_batch(self, dense: torch.Tensor, labels: torch.Tensor, offsets: torch.Tensor, values: torch.Tensor,
                  non_blocking: bool = True) -> None:
        self.dense_in.copy_(dense, non_blocking=non_blocking)
        self.labels.copy_(labels.reshape(-1), non_blocking=non_blocking)
        self.emb.set_input(offsets, values, non_blocking=non_blocking)

    # ------------------------------------------------------------------ step
    def _build_ops(self) -> None:
        """The training step as a flat list of (name, launch) pairs, in stream order."""
        C = native()
        ds = self.dense
        ops = [("emb.forward", lambda: self.emb.forward(training=True)),
               ("concat_x0", lambda: C.dcn_concat_x0(self.emb.pooled_output.data_ptr(), self.E, self.dense_in.data_ptr(),
                                                     self.cfg.num_dense, self.m, self.E, self.x0.local.data_ptr(),
                                                     self.x0.ld))]
        ops += self.fwd_calls
        head = dict(h=self.final_in.data_ptr(), ldh=self.H, H=self.H, relu_from=self.ldW,
                    w=ds.compute_view("head.w").data_ptr(), bias=ds.compute_view("head.b").data_ptr(),
                    labels=self.labels.data_ptr(), B=self.m, grad_scale=1.0 / self.global_B,
                    logits=self.logits.data_ptr(), dl=self.dl.data_ptr(), dh=self.dfin.local.data_ptr(),
                    lddh=self.H, loss_sum=self.loss_sum.data_ptr(), db=ds.grad_view("head.b").data_ptr())
        ops.append(("loss.zero", self.loss_sum.zero_))
        ops.append(("head", lambda: C.dcn_head(head)))
        ops.append(("head.dw", lambda: C.dcn_scaled_colsum(self.final_in.data_ptr(), self.H, self.dl.data_ptr(),
                                                           self.m, self.H, ds.grad_view("head.w").data_ptr())))
        first = True
        for calls in self.bwd_cross:
            for c in calls:
                if c[0] == "elem":
                    _, l, g_next = c
                    acc = 0 if first else 1
                    first = False
                    ops.append((f"bwd.cross{l}.elem", lambda l=l, g=g_next, acc=acc: C.dcn_cross_bwd_elem(
                        g.data_ptr(), g.stride(0), self.x0.local.data_ptr(), self.z[l].data_ptr(), self.ldW, self.m,
                        self.ldW, self.dz.data_ptr(), self.dx0.data_ptr(), self.ldW, acc,
                        ds.grad_view(f"cross{l}.b").data_ptr())))
                else:
                    ops.append(self._op(c))
        ops += [self._op(c) for c in self.bwd_deep]
        ops.append(("finalize_grad", lambda: C.dcn_finalize_grad(self.dx0.data_ptr(), self.ldW, self.m, self.E,
                                                                 self.emb.grad_input.data_ptr(),
                                                                 self.emb.grad_input.stride(0))))
        self.fb_ops = ops
        upd = [("emb.backward", self.emb.backward), ("dense.apply", self.dense.apply)]
        upd += [(f"fsdp.{w.name}", lambda w=w: w.apply(self.dense.step)) for w in self.fsdp_weights]
        self.update_ops = upd

    @staticmethod
    def _op(c):
        if isinstance(c[1], DistGemm):
            return c
        if c[0] == "wgrad":
            _, name, dy, x, out = c
            return name, lambda: gemm(dy, x, a_t=True, b_t=True, out=out, accumulate=True)
        if c[0] == "colsum":
            _, name, x, out = c
            return name, lambda: colsum_(x, out)
        raise ValueError(c[0])

    # ------------------------------------------------------------------ step
    def forward(self, training: bool = True) -> None:
        """Forward pass only (eval: ``training=False`` leaves the sparse staging untouched)."""
        C = native()
        pooled = self.emb.forward(training=training)
        C.dcn_concat_x0(pooled.data_ptr(), pooled.stride(0), self.dense_in.data_ptr(), self.cfg.num_dense, self.m,
                        self.E, self.x0.local.data_ptr(), self.x0.ld)
        for _, call in self.fwd_calls:
            call()

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
        """Run one eager training step with CUDA events between ops; returns (name, ms) per op."""
        evs = []
        ops = self.fb_ops + self.update_ops
        for name, op in ops:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append((name, e))
            op()
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        torch.cuda.synchronize()
        out = []
        for i, (name, e) in enumerate(evs):
            nxt = evs[i + 1][1] if i + 1 < len(evs) else end
            out.append((name, e.elapsed_time(nxt)))
        return out

    def check(self) -> None:
        self.emb.check()
        self.ctx.check("DCN GEMMs")
        if self.dense.status is not None:
            self.dense.status.check("dense optimizer")

    # ------------------------------------------------------------- export
    def logical_weights(self) -> dict[str, torch.Tensor]:
        """fp32 master weights of the logical model (collective when world > 1)."""
        import torch.distributed as dist

        cfg, tp = self.cfg, self.tp
        out = {}
        for l in range(cfg.cross_layers):
            out[f"cross{l}.V"] = self.V[l].gather_master().cpu()
            out[f"cross{l}.U"] = self.U[l].gather_master().cpu()
        for i, w in enumerate(self.deepW):
            shard = w.gather_master()
            if tp > 1:
                parts = [torch.empty_like(shard) for _ in range(self.world)]
                dist.all_gather(parts, shard.contiguous())
                tpp = [parts[r] for r in self.mesh.tp_group(self.rank)]
                shard = torch.cat(tpp, 0 if self.col_parallel[i] else 1)
            out[f"deep{i}.W"] = shard.cpu()
        master = self.dense.gather_master().cpu()
        for name, e in self.params.entries.items():
            out[name] = master[e.offset:e.offset + e.numel].reshape(e.shape).clone()
        hw = out["head.w"]
        out["head.w"] = torch.cat([hw[:self.W], hw[self.ldW:]])
        return out


# ---------------------------------------------------------------------------
# PyTorch reference / baseline
# ---------------------------------------------------------------------------
class DCNTorch(nn.Module):
    """DCN-v2 in plain PyTorch autograd (EmbeddingBag sum pooling, Linear layers)."""

    def __init__(self, cfg: DCNConfig, *, seed: int = 0, dtype: torch.dtype = torch.float32,
                 device: torch.device | str | None = None, sparse_grad: bool = False):
        super().__init__()
        self.cfg = cfg
        dk = {"device": device}
        self.embs = nn.ModuleList(nn.EmbeddingBag(t.num_embeddings, t.embedding_dim, mode="sum", sparse=sparse_grad,
                                                  **dk) for t in cfg.tables)
        W, r = cfg.width, cfg.cross_rank
        self.V = nn.ModuleList(nn.Linear(W, r, bias=False, **dk) for _ in range(cfg.cross_layers))
        self.U = nn.ModuleList(nn.Linear(r, W, **dk) for _ in range(cfg.cross_layers))
        dims = [W] + list(cfg.deep)
        self.deep = nn.ModuleList(nn.Linear(a, b, **dk) for a, b in zip(dims[:-1], dims[1:]))
        self.head = nn.Linear(W + cfg.deep[-1], 1, **dk)
        self.compute_dtype = dtype
        self.load_logical(dcn_init_weights(cfg, seed))

    @torch.no_grad()
    def load_logical(self, w: dict[str, torch.Tensor]) -> "DCNTorch":
        for l in range(self.cfg.cross_layers):
            self.V[l].weight.copy_(w[f"cross{l}.V"])
            self.U[l].weight.copy_(w[f"cross{l}.U"])
            self.U[l].bias.copy_(w[f"cross{l}.b"])
        for i, lin in enumerate(self.deep):
            lin.weight.copy_(w[f"deep{i}.W"])
            lin.bias.copy_(w[f"deep{i}.b"])
        self.head.weight.copy_(w["head.w"].reshape(1, -1))
        self.head.bias.copy_(w["head.b"])
        return self

    @torch.no_grad()
    def load_tables_from(self, fused: DCN) -> "DCNTorch":
        for i, s in enumerate(fused.emb.shards):
            self.embs[s.table].weight[s.row_slice, s.col_begin:s.col_begin + s.ncols] = fused.emb.shard_view(i).float().to(
                self.embs[s.table].weight.device)
        return self

    def pooled(self, offsets, values, B):
        outs = []
        offs, vals = offsets.long(), values.long()
        for f, e in enumerate(self.embs):
            beg = offs[f * B:(f + 1) * B + 1]
            outs.append(e(vals[beg[0]:beg[-1]], beg[:-1] - beg[0]))
        return torch.cat(outs, 1)

    def forward_from_pooled(self, pooled: torch.Tensor, dense: torch.Tensor) -> torch.Tensor:
        with torch.autocast(device_type=pooled.device.type, dtype=self.compute_dtype,
                            enabled=self.compute_dtype != torch.float32):
            x0 = torch.cat([pooled, dense.to(pooled.dtype)], 1)
            x = x0
            for V, U in zip(self.V, self.U):
                x = x0 * U(V(x)) + x
            h = x0
            for lin in self.deep:
                h = torch.relu(lin(h))
            return self.head(torch.cat([x, h], 1)).float().reshape(-1)

    def forward(self, dense, offsets, values):
        return self.forward_from_pooled(self.pooled(offsets, values, dense.shape[0]), dense)


__all__ = ["DCN", "DCNConfig", "DCNTorch", "dcn_benchmark_tables", "dcn_init_weights"]
