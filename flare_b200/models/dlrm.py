"""DLRM-style ranking model: B200 fused path and a plain PyTorch reference.

``DLRM`` (the product path) runs one training step as a fixed sequence of
hand-written sm_100a kernels on static buffers, so the whole step can be
captured in a CUDA graph:

    cast(dense) -> bottom MLP (tcgen05 GEMMs, bias+ReLU epilogues)
    sharded embedding forward (ids all-to-all + gather/pool + pooled all-to-all, one kernel)
    pairwise dot interaction -> top MLP -> fused head + BCE (fwd + bwd)
    top MLP backward (fused ReLU-mask / bias-grad epilogues) -> interaction backward
    bottom MLP backward -> sharded embedding backward (grad all-to-all + dedup + row-wise optimizer)
    dense optimizer (fused reduce-scatter + Adam + all-gather when data parallel)

With ``sparse_policy="pipelined"`` (the default when every table's
``max_staleness_steps`` is at least 1) the sparse update of step t-d runs in
the shadow of step t's dense work, d being the smallest
``max_staleness_steps`` of the tables (or ``staleness``): a side stream
carries every kernel that waits on the other ranks (embedding forward of
step t, embedding backward of step t-d, the dense update) in the same order
on every rank, while the main stream runs the dense kernels, which wait on
nothing.  Step t therefore looks up tables that lack the updates of steps
t-d .. t-1 (the reference's bounded-stale lookups with pipeline depth d + 1:
``sparse_lookup_async_policy``, src/flare/runtime/fluxway/workers/
dynamic_embedding.py:109-130, and ``AsyncPolicy.pipelined``, .../
sparse_input.py:473-476); staging and pooled-gradient buffers rotate over
d + 1 slots.  ``flush_pending_updates`` applies the pending updates in step
order (before a checkpoint, an evaluation or the end of training, as the
reference's ``flush_pending_updates``, .../dynamic_embedding.py:683).

``DLRMTorch`` is the same model in plain PyTorch autograd (nn.EmbeddingBag,
nn.Linear, torch optimizers): the CPU configuration, the numerics oracle and
the library baseline arm (cuBLAS + NCCL through DDP) of the benchmark.

The reference ships no concrete DLRM; applications build models from its MLP
and embedding layers (src/flare/jax/layers/base.py:27,
src/flare/jax/layers/embedding.py:13) and train them with row-wise sparse
optimizers in its external store (src/flare/runtime/fluxway/workers/
dynamic_embedding.py:69-106).
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import torch
import torch.nn as nn

from .._native import DeviceStatus
from ..ops.dense import cast_pad_bf16, head_bce, interaction_backward, interaction_forward, interaction_out_width
from ..parallel.symm import SymmetricHeap
from ..sparse.collection import ShardedEmbeddingBagCollection
from ..sparse.config import SparseOptimizerConfig, SparseTableSpec
from ..sparse.planner import ShardingPlan, plan_sharding
from ..training.flat import DenseOptimizerConfig, DenseState, FlatParams
from .mlp import MLPTower, pad_to


@dataclass
class DLRMConfig:
    tables: list[SparseTableSpec]
    num_dense: int = 13
    bottom: tuple[int, ...] = (512, 256, 128)
    top: tuple[int, ...] = (1024, 1024, 512, 256)
    num_targets: int = 1
    dense_optimizer: DenseOptimizerConfig = field(default_factory=DenseOptimizerConfig)
    sparse_optimizer: SparseOptimizerConfig = field(default_factory=SparseOptimizerConfig)

    def __post_init__(self):
        dims = {t.embedding_dim for t in self.tables}
        if dims != {self.bottom[-1]}:
            raise ValueError("every table's embedding_dim must equal the bottom MLP output width")

    @property
    def embedding_dim(self) -> int:
        return self.bottom[-1]

    @property
    def interaction_width(self) -> int:
        return interaction_out_width(len(self.tables), self.embedding_dim)

    def dense_flops_per_sample(self) -> float:
        """Forward+backward FLOPs of the dense part (GEMMs + interaction), per sample."""
        dims_b = [pad_to(self.num_dense)] + list(self.bottom)
        dims_t = [self.interaction_width] + list(self.top)
        f = sum(2 * a * b for a, b in zip(dims_b[:-1], dims_b[1:]))
        f += sum(2 * a * b for a, b in zip(dims_t[:-1], dims_t[1:]))
        T = len(self.tables) + 1
        f += 2 * T * T * self.embedding_dim // 2
        return 3.0 * f


def dlrm_benchmark_tables(vocab_sizes: list[int], dim: int = 128, optimizer: SparseOptimizerConfig | None = None,
                          value_dtype: str = "float32") -> list[SparseTableSpec]:
    opt = optimizer or SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.01)
    return [SparseTableSpec(f"t{i}", int(v), dim, optimizer=opt, value_dtype=value_dtype)
            for i, v in enumerate(vocab_sizes)]


MAX_PIPELINE_STALENESS = 4  # staging and pooled-gradient buffers per slot: d + 1 of each


def sparse_staleness(cfg: DLRMConfig, sparse_policy: str | None = None, staleness: int | None = None,
                     accumulation_steps: int = 1) -> int:
    """Steps of update lag the sparse policy runs with: 0 (sync) or d >= 1 (pipelined)."""
    stale = [t.max_staleness_steps for t in cfg.tables]
    if sparse_policy is None:  # from the tables: a staleness bound of >= 1 step everywhere allows the overlap
        sparse_policy = "pipelined" if stale and min(stale) >= 1 and accumulation_steps == 1 else "sync"
    if sparse_policy not in ("sync", "pipelined"):
        raise ValueError(f"sparse_policy must be 'sync' or 'pipelined', not {sparse_policy!r}")
    if sparse_policy == "sync":
        return 0
    if accumulation_steps > 1:
        raise ValueError("accumulation windows run under the sync sparse policy")
    d = int(staleness) if staleness is not None else max(1, min(stale, default=1))
    if not 1 <= d <= MAX_PIPELINE_STALENESS:
        raise ValueError(f"pipelined staleness must be in [1, {MAX_PIPELINE_STALENESS}], got {d}")
    if stale and d > min(stale) and min(stale) >= 1:
        raise ValueError(f"staleness {d} exceeds a table's max_staleness_steps ({min(stale)})")
    return d


def dlrm_plan(cfg: DLRMConfig, world_size: int, table_costs: list[float] | None = None, *,
              row_split: bool = False) -> ShardingPlan | None:
    """Sharding plan weighted by per-table work (None: the collection's default plan)."""
    if table_costs is None:
        return None
    tabs = [t if t.optimizer == cfg.sparse_optimizer else replace(t, optimizer=cfg.sparse_optimizer)
            for t in cfg.tables]
    return plan_sharding(tabs, world_size, expected_lookups=table_costs, row_split=row_split)


class DLRM:
    """Fused B200 DLRM for one rank's local batch."""

    def __init__(self, cfg: DLRMConfig, batch_size: int, *, max_bag_size: int, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, heap: SymmetricHeap | None = None, seed: int = 0,
                 global_batch_size: int | None = None, values_capacity: int | None = None,
                 table_costs: list[float] | None = None, plan: ShardingPlan | None = None,
                 sparse_policy: str | None = None, accumulation_steps: int = 1, staleness: int | None = None):
        self.accum = int(accumulation_steps)
        if self.accum < 1:
            raise ValueError("accumulation_steps must be >= 1")
        self.staleness = sparse_staleness(cfg, sparse_policy, staleness, self.accum)
        self.cfg = cfg
        self.pipelined = self.staleness > 0
        self.sparse_policy = "pipelined" if self.pipelined else "sync"
        self.B = int(batch_size)
        self.global_B = int(global_batch_size or batch_size * world_size)
        self.rank, self.world = rank, world_size
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        D = cfg.embedding_dim
        F = len(cfg.tables)
        self.F = F

        params = FlatParams()
        self.bottom = MLPTower("bottom", [cfg.num_dense] + list(cfg.bottom), params, relu_last=True)
        self.top = MLPTower("top", [cfg.interaction_width] + list(cfg.top), params, relu_last=True)
        H = cfg.top[-1]
        params.register("head.weight", (cfg.num_targets, H), "normal", (2.0 / (H + 1)) ** 0.5)
        params.register("head.bias", (cfg.num_targets,), "zeros")
        self.params = params
        self.dense = DenseState(params, cfg.dense_optimizer, device=dev, rank=rank, world_size=world_size,
                                heap=heap, seed=seed)
        self.bottom.bind(self.dense, self.B)
        self.top.bind(self.dense, self.B)
        self.head_w = self.dense.compute_view("head.weight")
        self.head_b = self.dense.compute_view("head.bias")
        self.head_dw = self.dense.grad_view("head.weight")
        self.head_db = self.dense.grad_view("head.bias")

        self.emb = ShardedEmbeddingBagCollection(
            cfg.tables, self.B, max_bag_size=max_bag_size, rank=rank, world_size=world_size, device=dev, heap=heap,
            optimizer=cfg.sparse_optimizer, seed=seed, values_capacity=values_capacity,
            plan=plan if plan is not None else dlrm_plan(cfg, world_size, table_costs), pipelined=self.pipelined,
            pipeline_depth=max(self.staleness, 1), accumulation_steps=self.accum)
        # pipelined policy: staging slot of the next forward; slots whose sparse updates are pending, oldest first
        self._next_slot = 0
        self.pending: list[int] = []
        if self.pipelined:
            # high priority: the side stream carries the step's critical path (embedding forward and
            # backward); the dense kernels beside it fill the SMs it leaves
            self.comm_stream = torch.cuda.Stream(device=dev, priority=-1)
            self._ev_fwd = torch.cuda.Event()
            self._ev_bwd = torch.cuda.Event()

        bf = dict(dtype=torch.bfloat16, device=dev)
        self.dense_in = torch.zeros(self.B, cfg.num_dense, dtype=torch.float32, device=dev)
        self.labels = torch.zeros(self.B, cfg.num_targets, dtype=torch.float32, device=dev)
        self.xd = torch.zeros(self.B, self.bottom.in_dim, **bf)
        self.inter = torch.zeros(self.B, cfg.interaction_width, **bf)
        self.dbot = torch.empty(self.B, D, **bf)
        self.dh = torch.empty(self.B, H, **bf)
        self.logits = torch.zeros(self.B, cfg.num_targets, dtype=torch.float32, device=dev)
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        self.inter_status = DeviceStatus(dev)  # bounded tensor-core waits of the interaction kernels

    # ------------------------------------------------------------------ data
    def set_batch(self, dense: torch.Tensor, labels: torch.Tensor, offsets: torch.Tensor, values: torch.Tensor,
                  non_blocking: bool = True) -> None:
        self.dense_in.copy_(dense, non_blocking=non_blocking)
        self.labels.copy_(labels.reshape(self.B, -1), non_blocking=non_blocking)
        self.emb.set_input(offsets, values, non_blocking=non_blocking)

    # ------------------------------------------------------------------ step
    def forward_backward(self) -> torch.Tensor:
        """Forward + backward of the local batch; gradients land in the flat/sparse buffers.

        Synchronous semantics: a sparse update still pending under the pipelined policy is applied
        first (its staging slot is the one this forward would reuse).  In an accumulation window the
        dense gradients add up in the flat buffer and the pooled gradients in the window's micro-step
        slot."""
        self._flush_pipelined()
        cast_pad_bf16(self.dense_in, self.xd, zero=self.loss_sum)  # also clears the loss accumulator
        bot = self.bottom.forward(self.xd)
        pooled = self.emb.forward()
        interaction_forward(bot, pooled, self.F, self.inter, self.inter_status)
        h = self.top.forward(self.inter)
        head_bce(h, self.head_w, self.head_b, self.labels, grad_scale=1.0 / self.global_B, logits=self.logits,
                 loss_sum=self.loss_sum, dh=self.dh, dw=self.head_dw, db=self.head_db)
        dinter = self.top.backward(self.dh, need_input_grad=True)
        interaction_backward(dinter, bot, pooled, self.F, self.dbot, self.emb.grad_input, relu_mask_bot=True,
                             status=self.inter_status)
        self.bottom.backward(self.dbot, need_input_grad=False)
        return self.loss_sum

    def profile_step(self) -> list[tuple[str, float]]:
        """One eager (synchronous) training step with CUDA events between its ops; returns (op, ms) in order."""
        self.flush_pending_updates()
        st: dict = {}

        def inter_fwd():
            interaction_forward(st["bot"], st["pooled"], self.F, self.inter, self.inter_status)

        def head():
            self.loss_sum.zero_()
            head_bce(st["h"], self.head_w, self.head_b, self.labels, grad_scale=1.0 / self.global_B,
                     logits=self.logits, loss_sum=self.loss_sum, dh=self.dh, dw=self.head_dw, db=self.head_db)

        def inter_bwd():
            interaction_backward(st["dinter"], st["bot"], st["pooled"], self.F, self.dbot, self.emb.grad_input,
                                 relu_mask_bot=True, status=self.inter_status)

        ops = [
            ("cast_dense", lambda: cast_pad_bf16(self.dense_in, self.xd)),
            ("bottom_fwd", lambda: st.__setitem__("bot", self.bottom.forward(self.xd))),
            ("emb_fwd", lambda: st.__setitem__("pooled", self.emb.forward())),
            ("interaction_fwd", inter_fwd),
            ("top_fwd", lambda: st.__setitem__("h", self.top.forward(self.inter))),
            ("head_bce", head),
            ("top_bwd", lambda: st.__setitem__("dinter", self.top.backward(self.dh, need_input_grad=True))),
            ("interaction_bwd", inter_bwd),
            ("bottom_bwd", lambda: self.bottom.backward(self.dbot, need_input_grad=False)),
            ("emb_bwd", lambda: self.emb.backward()),
            ("dense_apply", lambda: self.dense.apply()),
        ]
        evs = []
        for name, op in ops:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append((name, e))
            op()
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        torch.cuda.synchronize(self.device)
        return [(name, e.elapsed_time(evs[i + 1][1] if i + 1 < len(evs) else end)) for i, (name, e) in enumerate(evs)]

    def traced_step(self, tracer, step: int) -> torch.Tensor:
        """One eager training step that records the semantic execution trace (opt-in diagnostics).

        Emits one event per stage with the reference's stage names (input_unique, sparse_lookup,
        module_gather, module_gradient, sparse_update, module_update, sparse_commit; reference:
        recipes/recsys/ranking/metrics/execution_trace.py:75-380) carrying tensor summaries
        (finite / NaN / Inf counts, range, mean) and counters, inside NVTX ranges of the same names.
        Reading the summaries synchronises the device, so this is a diagnostics path, not the hot
        one; ``flare_b200.utils.trace_audit`` replays the trace."""
        nvtx = torch.cuda.nvtx
        self.flush_pending_updates()
        with nvtx.range("input_unique"):
            offs = self.emb.in_offsets.local
            nnz = int(offs[-1])
            tracer.emit("input_unique", "step", step=step, ids=nnz, bags=int(offs.numel() - 1),
                        values=self.emb.in_values.local[:nnz])
        with nvtx.range("sparse_lookup"):
            cast_pad_bf16(self.dense_in, self.xd)
            bot = self.bottom.forward(self.xd)
            pooled = self.emb.forward()
            tracer.emit("sparse_lookup", "step", step=step, pooled=pooled)
        with nvtx.range("module_gather"):
            interaction_forward(bot, pooled, self.F, self.inter, self.inter_status)
            tracer.emit("module_gather", "step", step=step, bottom=bot, interaction=self.inter)
        with nvtx.range("module_gradient"):
            h = self.top.forward(self.inter)
            self.loss_sum.zero_()
            head_bce(h, self.head_w, self.head_b, self.labels, grad_scale=1.0 / self.global_B, logits=self.logits,
                     loss_sum=self.loss_sum, dh=self.dh, dw=self.head_dw, db=self.head_db)
            dinter = self.top.backward(self.dh, need_input_grad=True)
            interaction_backward(dinter, bot, pooled, self.F, self.dbot, self.emb.grad_input, relu_mask_bot=True,
                                 status=self.inter_status)
            self.bottom.backward(self.dbot, need_input_grad=False)
            tracer.emit("module_gradient", "step", step=step, loss_sum=float(self.loss_sum), logits=self.logits,
                        dense_grad=self.dense.grad, sparse_input_grad=self.emb.grad_input)
        with nvtx.range("sparse_update"):
            self.emb.backward()
            tracer.emit("sparse_update", "step", step=step, **self.emb.last_step_stats())
        with nvtx.range("module_update"):
            self.dense.apply()
            tracer.emit("module_update", "step", step=step, master=self.dense.master)
        with nvtx.range("sparse_commit"):
            tracer.emit("sparse_commit", "step", step=step, sparse_optimizer_step=self.emb.step,
                        dense_optimizer_step=self.dense.step)
        return self.loss_sum

    def train_step(self) -> torch.Tensor:
        """One step; returns the device scalar sum of per-sample losses.

        With ``accumulation_steps`` n > 1 a call is one micro-step: the n-th call of a window applies
        the sparse and dense optimizers once to the window's summed gradients divided by n (the
        reference's micro-step windows with the update at the boundary:
        src/flare/jax/training/engines/distributed.py:1017-1180 and the sparse fp32 accumulation
        before ``optimizer_step(n_micro)``, src/flare/runtime/fluxway/workers/dynamic_embedding.py:
        481-549)."""
        if self.pipelined:
            return self._pipelined_step()
        loss = self.forward_backward()
        if self.accum == 1 or self.emb.micro_filled == self.accum:
            self._close_window()
        return loss

    def _close_window(self) -> None:
        micro = self.emb.micro_filled if self.accum > 1 else 1
        self.emb.backward()
        self.dense.apply(grad_scale=1.0 / micro)

    @property
    def pending_slot(self) -> int | None:
        """Slot of the newest pending sparse update (None when nothing is pending)."""
        return self.pending[-1] if self.pending else None

    def _pipelined_step(self) -> torch.Tensor:
        main = torch.cuda.current_stream(self.device)
        comm = self.comm_stream
        slot = self._next_slot
        pend = self.pending[0] if len(self.pending) == self.staleness else None
        comm.wait_stream(main)  # this step's inputs and the previous step's dense reads are ordered before
        cast_pad_bf16(self.dense_in, self.xd, zero=self.loss_sum)  # also clears the loss accumulator
        bot = self.bottom.forward(self.xd)
        with torch.cuda.stream(comm):
            pooled = self.emb.forward(slot=slot)
            self._ev_fwd.record(comm)
            if pend is not None:
                self.emb.backward(slot=pend)  # step t-d's sparse update, beside this step's dense work
        main.wait_event(self._ev_fwd)
        interaction_forward(bot, pooled, self.F, self.inter, self.inter_status)
        h = self.top.forward(self.inter)
        head_bce(h, self.head_w, self.head_b, self.labels, grad_scale=1.0 / self.global_B, logits=self.logits,
                 loss_sum=self.loss_sum, dh=self.dh, dw=self.head_dw, db=self.head_db)
        dinter = self.top.backward(self.dh, need_input_grad=True)
        interaction_backward(dinter, bot, pooled, self.F, self.dbot, self.emb.grad_ins[slot].local,
                             relu_mask_bot=True, status=self.inter_status)
        self.bottom.backward(self.dbot, need_input_grad=False)
        self._ev_bwd.record(main)
        with torch.cuda.stream(comm):
            comm.wait_event(self._ev_bwd)
            self.dense.apply()
        main.wait_stream(comm)
        self.pending = (self.pending[1:] if pend is not None else self.pending) + [slot]
        self._next_slot = (slot + 1) % (self.staleness + 1)
        return self.loss_sum

    def flush_pending_updates(self) -> bool:
        """Apply what the model holds back: the pending sparse update of the pipelined policy, or the
        open accumulation window (a tail window, normalised by its own micro-step count); True if
        there was something."""
        if self.accum > 1 and self.emb.micro_filled > 0:
            self._close_window()
            return True
        return self._flush_pipelined()

    def _flush_pipelined(self) -> bool:
        if not self.pending:
            return False
        for sl in self.pending:
            self.emb.backward(slot=sl)
        self.pending = []
        return True

    # host-side state of a step, for CUDA-graph capture (undone) and replay (advanced)
    def graph_key(self):
        """Steps with equal keys launch the same kernels on the same buffers (None: do not capture)."""
        if self.accum > 1:
            return ("micro", self.emb.micro_filled)
        if not self.pipelined:
            return 0
        # steps that fill the pipeline run eagerly; a full pipeline cycles through d + 1 states
        return None if len(self.pending) < self.staleness else (self._next_slot, tuple(self.pending))

    def host_state(self) -> tuple:
        return (self.dense.step, self.emb.step, self._next_slot, tuple(self.pending), self.emb._slot,
                self.emb.micro_filled, self.emb._micro)

    def restore_host_state(self, st: tuple) -> None:
        (self.dense.step, self.emb.step, self._next_slot, pending, self.emb._slot,
         self.emb.micro_filled, self.emb._micro) = st
        self.pending = list(pending)

    def advance_host_state(self) -> None:
        """The host-side effect of one replayed step (a captured step runs exactly one sparse backward:
        its own under the sync policy, the pending one under the pipelined policy; a micro-step of an
        accumulation window runs one only when it closes the window)."""
        if self.accum > 1:
            k = self.emb.micro_filled
            self.emb._micro = k
            if k + 1 < self.accum:
                self.emb.micro_filled = k + 1
                return
            self.emb.micro_filled = 0
        self.dense.step += 1
        self.emb.step += 1
        if self.pipelined:
            slot = self._next_slot
            self.emb._slot = slot
            self.pending = self.pending[1:] + [slot]
            self._next_slot = (slot + 1) % (self.staleness + 1)

    def predict(self) -> torch.Tensor:
        """Forward only (eval): sigmoid probabilities [B, T]; no state changes besides staging.

        Under the pipelined policy the pending sparse update is applied first, so the
        prediction sees every trained step."""
        self.flush_pending_updates()
        cast_pad_bf16(self.dense_in, self.xd)
        bot = self.bottom.forward(self.xd)
        pooled = self.emb.forward(training=False)
        interaction_forward(bot, pooled, self.F, self.inter, self.inter_status)
        h = self.top.forward(self.inter)
        x = h.float() @ self.head_w.float().t() + self.head_b.float()
        return torch.sigmoid(x)

    def check(self) -> None:
        self.emb.check()
        self.inter_status.check("dot interaction")
        if self.dense.status is not None:
            self.dense.status.check("dense optimizer")


# ---------------------------------------------------------------------------
# Plain PyTorch reference / baseline
# ---------------------------------------------------------------------------
class RowwiseAdagradTorch:
    """Row-wise Adagrad for ``nn.EmbeddingBag(sparse=True)`` tables in plain PyTorch.

    Per touched row r with summed gradient g_r (plus weight decay): state_r += mean(g_r^2) over the
    row's columns; w_r -= lr * g_r / (sqrt(state_r) + eps) -- the update of the fused kernels and of
    the reference's row-wise optimizer (src/flare/runtime/fluxway/workers/dynamic_embedding.py:481-549).
    ``all_gather_grads``: with replicated tables on several ranks, every rank applies the union of all
    ranks' sparse gradients, each divided by the world size (the global-mean gradient)."""

    def __init__(self, params, lr: float = 0.01, eps: float = 1e-8, weight_decay: float = 0.0,
                 all_gather_grads: bool = False):
        self.params = list(params)
        self.lr, self.eps, self.wd = float(lr), float(eps), float(weight_decay)
        self.state = [torch.zeros(p.shape[0], device=p.device) for p in self.params]
        self.gather = all_gather_grads

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None

    @torch.no_grad()
    def step(self) -> None:
        import torch.distributed as dist

        for p, st in zip(self.params, self.state):
            if p.grad is None:
                continue
            g = p.grad.coalesce()
            idx, val = g.indices()[0], g.values().float()
            if self.gather and dist.is_initialized() and dist.get_world_size() > 1:
                w = dist.get_world_size()
                n = torch.tensor([idx.numel()], device=idx.device)
                ns = [torch.zeros_like(n) for _ in range(w)]
                dist.all_gather(ns, n)
                m = int(max(int(x) for x in ns))
                pad_i = torch.full((m,), -1, dtype=idx.dtype, device=idx.device)
                pad_v = torch.zeros((m, val.shape[1]), device=val.device)
                pad_i[:idx.numel()], pad_v[:idx.numel()] = idx, val
                gi = [torch.empty_like(pad_i) for _ in range(w)]
                gv = [torch.empty_like(pad_v) for _ in range(w)]
                dist.all_gather(gi, pad_i)
                dist.all_gather(gv, pad_v)
                allv = torch.cat(gv) / w
                alli = torch.cat(gi)
                keep = alli >= 0
                g = torch.sparse_coo_tensor(alli[keep].unsqueeze(0), allv[keep], p.shape).coalesce()
                idx, val = g.indices()[0], g.values()
            rows = p.data[idx].float()
            if self.wd:
                val = val + self.wd * rows
            st.index_add_(0, idx, (val * val).mean(1))
            scale = self.lr / (st[idx].sqrt() + self.eps)
            p.data[idx] = (rows - scale.unsqueeze(1) * val).to(p.dtype)


class DLRMTorch(nn.Module):
    """DLRM in plain PyTorch: nn.EmbeddingBag (sum), nn.Linear towers, dot interaction."""

    def __init__(self, cfg: DLRMConfig, *, dtype: torch.dtype = torch.float32, sparse_grad: bool = True):
        super().__init__()
        self.cfg = cfg
        D = cfg.embedding_dim
        self.embs = nn.ModuleList(
            nn.EmbeddingBag(t.num_embeddings, t.embedding_dim, mode=t.pooling, sparse=sparse_grad)
            for t in cfg.tables)
        for e, t in zip(self.embs, cfg.tables):
            nn.init.uniform_(e.weight, -t.init_scale, t.init_scale)

        def mlp(dims):
            layers = []
            for a, b in zip(dims[:-1], dims[1:]):
                layers += [nn.Linear(a, b), nn.ReLU()]
            return nn.Sequential(*layers)

        self.bottom = mlp([cfg.num_dense] + list(cfg.bottom))
        T = len(cfg.tables) + 1
        self.npairs = T * (T - 1) // 2
        self.top = mlp([D + self.npairs] + list(cfg.top))
        self.head = nn.Linear(cfg.top[-1], cfg.num_targets)
        ii, jj = torch.tril_indices(T, T, offset=-1)
        self.register_buffer("ii", ii, persistent=False)
        self.register_buffer("jj", jj, persistent=False)
        self.compute_dtype = dtype

    @torch.no_grad()
    def load_from_fused(self, fused: "DLRM") -> "DLRMTorch":
        """Copy the fused model's compute weights and (exported) tables into this module."""
        ds = fused.dense

        def copy_tower(seq, tower):
            lin = [m for m in seq if isinstance(m, nn.Linear)]
            for layer, wn, bn in zip(lin, tower.wnames, tower.bnames):
                w = ds.compute_view(wn).float()
                layer.weight.copy_(w[:, :layer.weight.shape[1]])
                layer.bias.copy_(ds.compute_view(bn).float())

        copy_tower(self.bottom, fused.bottom)
        copy_tower(self.top, fused.top)
        self.head.weight.copy_(ds.compute_view("head.weight").float())
        self.head.bias.copy_(ds.compute_view("head.bias").float())
        for i, s in enumerate(fused.emb.shards):
            self.embs[s.table].weight[s.row_slice, s.col_begin:s.col_begin + s.ncols] = fused.emb.shard_view(i).float().to(
                self.embs[s.table].weight.device)
        return self

    def pooled(self, offsets: torch.Tensor, values: torch.Tensor, B: int) -> torch.Tensor:
        outs = []
        offs = offsets.long()
        vals = values.long()
        for f, e in enumerate(self.embs):
            beg = offs[f * B:(f + 1) * B + 1]
            ids = vals[beg[0]:beg[-1]]
            outs.append(e(ids, beg[:-1] - beg[0]))
        return torch.stack(outs, 1)

    def forward(self, dense: torch.Tensor, offsets: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        B = dense.shape[0]
        with torch.autocast(device_type=dense.device.type, dtype=self.compute_dtype,
                            enabled=self.compute_dtype != torch.float32):
            bot = self.bottom(dense)
            emb = self.pooled(offsets, values, B).to(bot.dtype)
            z = torch.cat([bot.unsqueeze(1), emb], 1)
            zz = torch.bmm(z, z.transpose(1, 2))
            inter = torch.cat([bot, zz[:, self.ii, self.jj]], 1)
            h = self.top(inter)
            return self.head(h).float()


__all__ = ["RowwiseAdagradTorch", "DLRM", "DLRMConfig", "DLRMTorch", "dlrm_benchmark_tables"]
