"""Public training API for the fused models (DLRM, DCN-v2).

``DLRMTrainer.train_step(batch)`` is the call a user makes: it copies the
step's inputs from (pinned) host memory to the device, runs the fused training
step (replayed from a CUDA graph after the first call when ``use_graph``), and
returns the step's loss read back to the host.  ``train_step_async`` overlaps
the next batch's host->device copy with the current step on a side stream and
returns the loss of the previous step (one-step lag), which is how a
throughput-oriented loop uses it.

The reference drives the same phases through Fluxway operators
(recipes/recsys/ranking/workers/train_worker.py:271-664: prepare_sparse_
materialize -> prepare_jax_bind -> train_core -> scatter_sparse_grads ->
update -> materialize_train_metrics); ``prepare_execution`` there AOT-compiles
per signature, here it captures a CUDA graph per static shape.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .._native import native
from ..data.synthetic import SparseBatch
from ..models.dlrm import DLRM, DLRMConfig, dlrm_plan, sparse_staleness
from ..parallel.dist import barrier
from ..parallel.symm import SymmetricHeap
from ..sparse.collection import ShardedEmbeddingBagCollection


@dataclass
class StepResult:
    loss: float
    step: int


class FusedTrainer:
    """Step driver shared by the fused models (``DLRM``, ``DCN``).

    The model provides ``set_batch``, ``train_step`` (one optimizer step on
    static buffers, returning the device loss sum), ``loss_sum``, ``dense``
    and ``emb`` (whose host step mirrors advance once per step) and ``check``.
    """

    def __init__(self, model, batch_size: int, *, device: torch.device, rank: int = 0, world_size: int = 1,
                 use_graph: bool = True):
        self.device = device
        self.rank, self.world = rank, world_size
        self.B = batch_size
        self.model = model
        self.use_graph = use_graph
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graphs: dict = {}  # graph key of the model's host state -> captured step
        self.launches_per_step: int | None = None
        self.steps = 0
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self._staged: list[SparseBatch] = []
        self._stage_idx = 0
        self._loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        self._loss_event = [torch.cuda.Event(), torch.cuda.Event()]
        self._copy_done = torch.cuda.Event()
        self._stage_free = [torch.cuda.Event(), torch.cuda.Event()]
        self._stage_used = [False, False]
        self._pending = False
        if world_size > 1:
            # every rank finishes building (allocation, table init) before any
            # rank can enter a fused kernel that waits on its peers
            torch.cuda.synchronize(self.device)
            barrier()


    # ---------------------------------------------------------------- graph
    EAGER_STEPS = 2  # steps run eagerly (module load, allocator warm-up) before capture

    def _graph_key(self):
        f = getattr(self.model, "graph_key", None)
        return 0 if f is None else f()

    def _host_state(self):
        f = getattr(self.model, "host_state", None)
        return f() if f is not None else (self.model.dense.step, self.model.emb.step)

    def _restore_host_state(self, st) -> None:
        f = getattr(self.model, "restore_host_state", None)
        if f is not None:
            f(st)
        else:
            self.model.dense.step, self.model.emb.step = st

    def _advance_host_state(self) -> None:
        f = getattr(self.model, "advance_host_state", None)
        if f is not None:
            f()
        else:
            self.model.dense.step += 1
            self.model.emb.step += 1

    def prepare_execution(self) -> None:
        """Capture the training step of the model's current host state as a CUDA graph.

        Capture records kernels without running them, so it changes no state
        (the host-side mirrors the recording advanced are put back); the first
        replay performs the step.  Step counters used by the optimizers are
        device-resident and advance inside the graph.  A model whose steps
        alternate buffers (the pipelined sparse policy) gets one graph per key.
        """
        key = self._graph_key()
        if not self.use_graph or key is None or key in self.graphs:
            return
        torch.cuda.synchronize(self.device)
        st = self._host_state()
        before = native().launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.model.train_step()
        self.launches_per_step = native().launch_count() - before
        self._restore_host_state(st)
        self.graphs[key] = g
        self.graph = g

    def _run_step(self) -> torch.Tensor:
        if self.use_graph and self.steps >= self.EAGER_STEPS:
            self.prepare_execution()
        g = self.graphs.get(self._graph_key()) if self.use_graph else None
        if g is not None:
            g.replay()
            self._advance_host_state()
            return self.model.loss_sum
        before = native().launch_count()
        loss = self.model.train_step()
        self.launches_per_step = native().launch_count() - before
        return loss

    # ------------------------------------------------------------------ API
    def train_step(self, batch: SparseBatch) -> StepResult:
        """Copy ``batch`` (host or device) in, run one step, return the loss (host float)."""
        m = self.model
        m.set_batch(batch.dense, batch.labels, batch.offsets, batch.values, non_blocking=True)
        loss = self._run_step()
        self.steps += 1
        return StepResult(float(loss.item()) / self.B, self.steps)

    def train_step_async(self, batch: SparseBatch) -> StepResult | None:
        """Pipelined step: H2D of this batch overlaps the previous step; returns the previous step's loss."""
        m = self.model
        cur = torch.cuda.current_stream(self.device)
        if not self._staged:
            self._staged = [self._alloc_stage(batch) for _ in range(2)]
        idx = self._stage_idx
        stage = self._staged[idx]
        self._stage_idx ^= 1
        with torch.cuda.stream(self.copy_stream):
            if self._stage_used[idx]:
                # do not overwrite a stage until the step that read it has copied it out
                self.copy_stream.wait_event(self._stage_free[idx])
            for dst, src in zip((stage.dense, stage.labels, stage.offsets), (batch.dense, batch.labels, batch.offsets)):
                dst.copy_(src, non_blocking=True)
            stage.values[:batch.values.numel()].copy_(batch.values, non_blocking=True)
            self._copy_done.record(self.copy_stream)
        prev = None
        if self._pending:
            ev = self._loss_event[self.steps % 2]
            ev.synchronize()
            prev = StepResult(float(self._loss_host[self.steps % 2]) / self.B, self.steps)
        cur.wait_event(self._copy_done)
        m.set_batch(stage.dense, stage.labels, stage.offsets, stage.values[:batch.values.numel()], non_blocking=True)
        self._stage_free[idx].record(cur)
        self._stage_used[idx] = True
        loss = self._run_step()
        self.steps += 1
        slot = self.steps % 2
        self._loss_host[slot:slot + 1].copy_(loss, non_blocking=True)
        self._loss_event[slot].record(cur)
        self._pending = True
        return prev

    def flush(self) -> StepResult | None:
        if not self._pending:
            return None
        slot = self.steps % 2
        self._loss_event[slot].synchronize()
        self._pending = False
        return StepResult(float(self._loss_host[slot]) / self.B, self.steps)

    def _alloc_stage(self, batch: SparseBatch) -> SparseBatch:
        dev = self.device
        return SparseBatch(torch.empty_like(batch.dense, device=dev), torch.empty_like(batch.labels, device=dev),
                           torch.empty_like(batch.offsets, device=dev),
                           torch.empty(self.model.emb.values_capacity, dtype=torch.int32, device=dev))

    def check(self) -> None:
        self.model.check()

    def flush_pending_updates(self) -> bool:
        """Apply a sparse update the model still holds back (pipelined policy); True if there was one."""
        f = getattr(self.model, "flush_pending_updates", None)
        return bool(f()) if f is not None else False

    def close(self) -> None:
        self.flush_pending_updates()
        self.graph = None
        self.graphs.clear()
        torch.cuda.synchronize(self.device)


class DLRMTrainer(FusedTrainer):
    def __init__(self, cfg: DLRMConfig, batch_size: int, *, max_bag_size: int, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, seed: int = 0, use_graph: bool = True,
                 values_capacity: int | None = None, heap_bytes: int | None = None,
                 table_costs: list[float] | None = None, row_split: bool = False, sparse_policy: str | None = None,
                 accumulation_steps: int = 1, staleness: int | None = None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        heap = None
        plan = dlrm_plan(cfg, world_size, table_costs, row_split=row_split)
        depth = sparse_staleness(cfg, sparse_policy, staleness, accumulation_steps)
        if world_size > 1:
            exchange = ShardedEmbeddingBagCollection.exchange_bytes(
                cfg.tables, batch_size, max_bag_size, values_capacity, plan=plan, pipelined=depth > 0,
                pipeline_depth=max(depth, 1), accumulation_steps=accumulation_steps)
            dense = 6 * 16 * 1024 * 1024  # flat fp32 grads + bf16 params for up to 16M parameters
            need = heap_bytes or (exchange + dense + 64 * 1024 * 1024)
            heap = SymmetricHeap(need, rank=rank, world_size=world_size, device=device)
        self.heap = heap
        model = DLRM(cfg, batch_size, max_bag_size=max_bag_size, rank=rank, world_size=world_size,
                     device=device, heap=heap, seed=seed, values_capacity=values_capacity, plan=plan,
                     sparse_policy=sparse_policy, accumulation_steps=accumulation_steps, staleness=staleness)
        super().__init__(model, batch_size, device=device, rank=rank, world_size=world_size, use_graph=use_graph)


class DCNTrainer(FusedTrainer):
    """Public training API of the fused DCN-v2 (tensor-parallel x FSDP) model."""

    def __init__(self, cfg, batch_size: int, *, max_bag_size: int, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, seed: int = 0, use_graph: bool = True,
                 values_capacity: int | None = None):
        from ..models.dcn import DCN

        device = device or torch.device("cuda", torch.cuda.current_device())
        model = DCN(cfg, batch_size, max_bag_size=max_bag_size, rank=rank, world_size=world_size, device=device,
                    seed=seed, values_capacity=values_capacity)
        self.heap = model.heap
        super().__init__(model, batch_size, device=device, rank=rank, world_size=world_size, use_graph=use_graph)


class SeqRecTrainer(FusedTrainer):
    """Public training API of the fused sequential-recommendation model (inputs: ``SeqBatch``)."""

    def __init__(self, cfg, nseq: int, T_cap: int, *, rank: int = 0, world_size: int = 1,
                 device: torch.device | None = None, seed: int = 0, use_graph: bool = True,
                 values_capacity: int | None = None):
        from ..models.seqrec import SeqRec

        device = device or torch.device("cuda", torch.cuda.current_device())
        model = SeqRec(cfg, nseq, T_cap, rank=rank, world_size=world_size, device=device, seed=seed,
                       values_capacity=values_capacity)
        self.heap = model.heap
        super().__init__(model, nseq, device=device, rank=rank, world_size=world_size, use_graph=use_graph)
        self._seq_stage = None
        self._nv = [1, 1]  # global token count of the step whose loss sits in each loss slot

    @staticmethod
    def _loss(v: float, num_valid: int) -> float:
        # loss_sum is this rank's sum of token losses; report it per token of the step's global count
        return v / max(float(num_valid), 1.0)

    def train_step(self, batch) -> StepResult:
        self.model.set_batch(batch, non_blocking=True)
        loss = self._run_step()
        self.steps += 1
        return StepResult(self._loss(float(loss.item()), int(batch.num_valid.reshape(-1)[0])), self.steps)

    def train_step_async(self, batch) -> StepResult | None:
        """H2D of ``batch`` on a side stream overlapping the previous step; returns the previous step's loss."""
        m = self.model
        cur = torch.cuda.current_stream(self.device)
        fields = ("seq_offsets", "target_row", "emb_offsets", "emb_values", "num_valid")
        if self._seq_stage is None:
            cap = m.emb.values_capacity
            self._seq_stage = [
                {f: (torch.empty(cap, dtype=torch.int32, device=self.device) if f == "emb_values"
                     else torch.empty_like(getattr(batch, f), device=self.device)) for f in fields}
                for _ in range(2)]
        idx = self._stage_idx
        st = self._seq_stage[idx]
        self._stage_idx ^= 1
        with torch.cuda.stream(self.copy_stream):
            if self._stage_used[idx]:
                self.copy_stream.wait_event(self._stage_free[idx])
            for f in fields:
                src = getattr(batch, f)
                st[f][:src.numel()].copy_(src, non_blocking=True)
            self._copy_done.record(self.copy_stream)
        prev = None
        if self._pending:
            ev = self._loss_event[self.steps % 2]
            ev.synchronize()
            prev = StepResult(self._loss(float(self._loss_host[self.steps % 2]), self._nv[self.steps % 2]),
                              self.steps)
        cur.wait_event(self._copy_done)
        from ..data.synthetic import SeqBatch

        staged = SeqBatch(st["seq_offsets"], st["target_row"], st["emb_offsets"],
                          st["emb_values"][:batch.emb_values.numel()], st["num_valid"], batch.tokens)
        m.set_batch(staged, non_blocking=True)
        self._stage_free[idx].record(cur)
        self._stage_used[idx] = True
        loss = self._run_step()
        self.steps += 1
        slot = self.steps % 2
        self._nv[slot] = int(batch.num_valid.reshape(-1)[0])
        self._loss_host[slot:slot + 1].copy_(loss, non_blocking=True)
        self._loss_event[slot].record(cur)
        self._pending = True
        return prev

    def flush(self) -> StepResult | None:
        if not self._pending:
            return None
        slot = self.steps % 2
        self._loss_event[slot].synchronize()
        self._pending = False
        return StepResult(self._loss(float(self._loss_host[slot]), self._nv[slot]), self.steps)



__all__ = ["DCNTrainer", "DLRMTrainer", "FusedTrainer", "SeqRecTrainer", "StepResult"]
