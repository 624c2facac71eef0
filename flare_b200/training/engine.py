"""Generic training engine for autograd models (micro-steps, ZeRO, checkpoints).

Behaviour follows the reference's distributed engine
(src/flare/jax/training/engines/distributed.py:187-1301) and its ZeRO
collectives (src/flare/jax/training/zero/collectives.py:14-95):

* every dense parameter lives in one flat fp32 master buffer, padded to a
  multiple of the ZeRO world size (state layout of
  src/flare/jax/training/state/layout.py:12-105);
* a training window has ``plan.accumulation.micro_steps`` micro-steps; with
  ``sync_mode="micro"`` gradients are reduced every micro-step, with
  ``"boundary"`` once per window;
* ZeRO-0 all-reduces and updates everywhere; ZeRO-1 all-reduces and updates
  the local optimizer shard, then all-gathers parameters; ZeRO-2 and ZeRO-3
  reduce-scatter; ZeRO-3 additionally keeps only the parameter shard between
  steps and all-gathers it before each micro-step;
* gradients travel in the precision policy's transport dtype (bf16 under
  mixed precision) and are averaged over the world size;
* ``shard_scope="node"`` shards the optimizer state (and, for ZeRO-2/3, the
  gradients and parameters) over the ranks of one node only: gradients are
  all-reduced over every rank and each rank keeps its node-local slice, and
  parameter shards are all-gathered inside the node (the node scope of
  src/flare/jax/training/zero/collectives.py:33-36), so the inter-node
  traffic is one all-reduce and the shards replicate across nodes;
* sharded optimizers must be elementwise (no global-norm clipping), the
  shard-update capability rule of
  src/flare/jax/training/optimizers/base.py:70-150;
* checkpoint capture is allowed only at a window boundary and stores logical
  (unpadded) shapes; ``finalize_checkpoint_window`` applies a partial window;
* non-parameter state (module buffers) follows the reference's rules
  (src/flare/jax/training/engines/distributed.py:663-701): float buffers
  (e.g. normalisation statistics) are averaged over the ranks after every
  micro-step, integer / bool buffers must stay replicated (checked against
  every rank's copy when ``check_replication``), the reported loss is the
  mean over the ranks, and the buffers are part of the checkpoint.

The B200 product paths (fused DLRM) do not use this engine's NCCL
collectives; they use the fused kernels of ``flare_b200.training.flat``.
This engine serves generic models, the CPU configuration and tests.
"""
from __future__ import annotations

import hashlib
import os
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from .contracts import OptimizerUpdateWindow, TrainingExecutionPlan, ZeroStage
from .flat import DenseOptimizerConfig, adam_reference
from .precision import PrecisionPolicy


@dataclass
class TrainStepResult:
    loss: float | torch.Tensor
    micro_step: int
    step: int
    optimizer_applied: bool
    outputs: Any = None


class TrainEngine:
    def __init__(self, model: nn.Module, loss_fn: Callable[[Any, Any], torch.Tensor], plan: TrainingExecutionPlan,
                 optimizer: DenseOptimizerConfig, *, precision: PrecisionPolicy = PrecisionPolicy.FP32,
                 process_group: dist.ProcessGroup | None = None, device: torch.device | None = None,
                 forward: Callable[[nn.Module, Any], Any] | None = None, node_size: int | None = None,
                 sync_buffers: bool = True, check_replication: bool = False, validate_constants: bool = False):
        self.model = model
        self.loss_fn = loss_fn
        self.plan = plan
        self.opt = optimizer
        self.precision = precision
        self.pg = process_group
        self.device = device or next(model.parameters()).device
        self.forward_fn = forward or (lambda m, x: m(x))
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.stage = plan.zero.stage
        if self.world > 1 and self.stage is not ZeroStage.REPLICATED and not optimizer.shardable:
            raise ValueError("sharded optimizer updates require an elementwise optimizer without global-norm clip")
        # shard group: every rank (global scope) or the ranks of this node (node scope)
        self.node_scope = plan.zero.shard_scope == "node" and self.world > 1
        self.shard_pg, q, shard_rank = self.pg, max(self.world, 1), self.rank
        if self.node_scope:
            ns = int(node_size or os.environ.get("LOCAL_WORLD_SIZE", self.world))
            if ns < 1 or self.world % ns:
                raise ValueError(f"node size {ns} does not divide the world size {self.world}")
            base = dist.get_process_group_ranks(process_group) if process_group is not None else list(range(self.world))
            for n in range(self.world // ns):  # every rank creates every node group, in the same order
                g = dist.new_group(base[n * ns:(n + 1) * ns])
                if n == self.rank // ns:
                    self.shard_pg = g
            q, shard_rank = ns, self.rank % ns
        self.shards = q
        self.micro_steps = plan.accumulation.micro_steps
        self.micro_step = 0
        self.step = 0
        self.params = [p for p in model.parameters() if p.requires_grad]
        self.names = [n for n, p in model.named_parameters() if p.requires_grad]
        self.sync_buffers, self.check_replication = sync_buffers, check_replication
        from .precision import constant_buffers

        self.constants = constant_buffers(model)  # immutable buffers: never averaged; checked on request
        self.validate_constants = validate_constants
        self.offsets, off = [], 0
        for p in self.params:
            self.offsets.append(off)
            off += p.numel()
        self.numel = off
        self.padded = (off + q - 1) // q * q
        self.shard = self.padded // q
        self.lo, self.hi = shard_rank * self.shard, (shard_rank + 1) * self.shard
        flat = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                flat[o:o + p.numel()] = p.detach().reshape(-1).float()
        if self.world > 1:  # every rank starts from rank 0's parameters
            dist.broadcast(flat, src=0, group=self.pg)
        owns_full = self.stage in (ZeroStage.REPLICATED,) or self.world == 1
        self.master = flat if owns_full else flat[self.lo:self.hi].clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.acc_grad = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        self.reduced = torch.zeros(self.padded if owns_full or self.stage is ZeroStage.OPTIMIZER_STATE else self.shard,
                                   dtype=torch.float32, device=self.device)
        self._scatter_params(flat)
        self.last_loss: float | None = None

    # ------------------------------------------------------------ helpers
    def _scatter_params(self, flat: torch.Tensor) -> None:
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                p.copy_(flat[o:o + p.numel()].view_as(p).to(p.dtype))

    def _gather_flat_grad(self) -> torch.Tensor:
        g = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        for p, o in zip(self.params, self.offsets):
            if p.grad is not None:
                g[o:o + p.numel()] = p.grad.reshape(-1).float()
        return g

    def _reduce(self, g: torch.Tensor) -> torch.Tensor:
        """Sum over ranks in the transport dtype, averaged; full or shard per stage."""
        if self.world == 1:
            return g
        wire = g.to(self.precision.gradient_transport_dtype)
        if self.stage in (ZeroStage.REPLICATED, ZeroStage.OPTIMIZER_STATE):
            dist.all_reduce(wire, group=self.pg)
            return wire.float() / self.world
        if self.node_scope:  # global sum, then this rank's node-local slice
            dist.all_reduce(wire, group=self.pg)
            return wire[self.lo:self.hi].float() / self.world
        out = torch.empty(self.shard, dtype=wire.dtype, device=self.device)
        dist.reduce_scatter_tensor(out, wire, group=self.pg)
        return out.float() / self.world

    def _materialize_params(self) -> None:
        """ZeRO-3: all-gather the parameter shards before a micro-step."""
        if self.world > 1 and self.stage is ZeroStage.PARAMETER:
            full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
            dist.all_gather_into_tensor(full, self.master, group=self.shard_pg)
            self._scatter_params(full)

    # --------------------------------------------------------------- step
    def micro_step_once(self, inputs: Any, targets: Any) -> TrainStepResult:
        if self.micro_step == 0:
            self._materialize_params()
        for p in self.params:
            p.grad = None
        dt = self.precision.compute_dtype
        before = {n: c.detach().clone() for n, c in self.constants.items()} if self.validate_constants else None
        with torch.autocast(device_type=self.device.type, dtype=dt, enabled=dt != torch.float32):
            outputs = self.forward_fn(self.model, inputs)
            loss = self.loss_fn(outputs, targets)
        loss.backward()
        if before is not None:
            for n, c in self.constants.items():
                if not torch.equal(before[n], c):
                    raise RuntimeError(f"constant buffer {n} changed during the forward / backward")
        self._sync_buffer_state()
        g = self._gather_flat_grad()
        self.micro_step += 1
        if self.plan.accumulation.sync_mode == "micro":
            r = self._reduce(g)
            self.reduced += r
        else:
            self.acc_grad += g
        at_boundary = self.micro_step == self.micro_steps
        applied = False
        if at_boundary and self.plan.update.apply_optimizer_at_boundary:
            self.apply_accumulated_update()
            applied = True
        mean_loss = loss.detach()
        if self.world > 1:  # the reported loss is the mean over the ranks
            mean_loss = mean_loss.float().clone()
            dist.all_reduce(mean_loss, group=self.pg)
            mean_loss = mean_loss / self.world
        self.last_loss = float(mean_loss)
        return TrainStepResult(mean_loss, self.micro_step if not applied else self.micro_steps, self.step,
                               at_boundary, outputs)

    def _sync_buffer_state(self) -> None:
        """Average float buffers over the ranks; check that the others are replicated (when asked)."""
        if self.world == 1 or not self.sync_buffers:
            return
        for name, b in self.model.named_buffers():
            if name in self.constants:
                continue
            if b.is_floating_point():
                t = b.detach().float().clone()
                dist.all_reduce(t, group=self.pg)
                b.copy_((t / self.world).to(b.dtype))
            elif self.check_replication:
                parts = [torch.empty_like(b) for _ in range(self.world)]
                dist.all_gather(parts, b.detach().contiguous(), group=self.pg)
                if any(not torch.equal(parts[0], x) for x in parts[1:]):
                    raise RuntimeError(f"non-float buffer {name} differs across ranks")

    def input_gradients(self, inputs: Mapping[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        """Gradients of the named inputs of the last micro-step (the pooled embeddings, for the sparse
        tables), normalised by world size x micro-steps: the sample-mean contract of
        ``training.gradients.normalize_input_gradients``."""
        from .gradients import input_gradients

        return input_gradients(inputs, world_size=self.world, micro_steps=self.micro_steps)

    def apply_accumulated_update(self, micro_steps: int | None = None) -> None:
        n = micro_steps or self.micro_steps
        if self.plan.accumulation.sync_mode == "boundary":
            self.reduced = self._reduce(self.acc_grad)
        g = self.reduced / n
        if self.stage is ZeroStage.OPTIMIZER_STATE and self.world > 1:
            g = g[self.lo:self.hi]
        self.step += 1
        op = self.opt.kernel_params(self.step)
        if self.opt.global_norm_clip is not None:
            norm = float(torch.linalg.vector_norm(g))
            if norm > self.opt.global_norm_clip:
                g = g * (self.opt.global_norm_clip / (norm + 1e-6))
        adam_reference(self.master, g, self.m, self.v, op)
        if self.world > 1 and self.stage is not ZeroStage.REPLICATED:
            full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
            dist.all_gather_into_tensor(full, self.master, group=self.shard_pg)
            self._scatter_params(full)
        else:
            self._scatter_params(self.master)
        self.acc_grad.zero_()
        self.reduced.zero_()
        self.micro_step = 0

    def finalize_checkpoint_window(self) -> bool:
        """Apply a partial window (actual length) before a checkpoint; True if applied."""
        if self.micro_step == 0:
            return False
        self.apply_accumulated_update(self.micro_step)
        return True

    # ----------------------------------------------------------- checkpoint
    def _full_master(self) -> torch.Tensor:
        if self.world == 1 or self.stage is ZeroStage.REPLICATED:
            return self.master
        full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, self.master, group=self.shard_pg)
        return full

    def _full(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1 or self.stage is ZeroStage.REPLICATED:
            return t
        full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, t, group=self.shard_pg)
        return full

    def _unflatten(self, flat: torch.Tensor) -> dict[str, torch.Tensor]:
        return {n: flat[o:o + p.numel()].view(p.shape).detach().cpu().clone()
                for n, p, o in zip(self.names, self.params, self.offsets)}

    def checkpoint_layout(self) -> Mapping[str, Any]:
        return {"leaves": [(n, tuple(p.shape), "float32") for n, p in zip(self.names, self.params)],
                "schema_digest": self.schema_digest(), "zero_stage": int(self.stage), "world_size": self.world,
                "shard_scope": "node" if self.node_scope else "global", "shards": self.shards}

    def schema_digest(self) -> str:
        h = hashlib.sha256()
        for n, p in zip(self.names, self.params):
            h.update(f"{n}:{tuple(p.shape)}:float32;".encode())
        return h.hexdigest()

    def capture_checkpoint_state(self) -> dict[str, Any]:
        if self.micro_step != 0:
            raise RuntimeError("checkpoint capture requires an optimizer-window boundary")
        return {"step": self.step, "schema_digest": self.schema_digest(),
                "model_state": self._unflatten(self._full_master()),
                "optimizer_state": {"m": self._unflatten(self._full(self.m)), "v": self._unflatten(self._full(self.v))},
                "buffers": {n: b.detach().cpu().clone() for n, b in self.model.named_buffers()}}

    def restore_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        if state.get("schema_digest") not in (None, self.schema_digest()):
            raise ValueError("checkpoint schema does not match this model")

        def flat_of(d):
            f = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
            for n, p, o in zip(self.names, self.params, self.offsets):
                t = d[n]
                if tuple(t.shape) != tuple(p.shape):
                    raise ValueError(f"checkpoint leaf {n} has shape {tuple(t.shape)}, expected {tuple(p.shape)}")
                f[o:o + p.numel()] = t.reshape(-1).to(self.device, torch.float32)
            return f

        owns_full = self.world == 1 or self.stage is ZeroStage.REPLICATED
        sl = slice(None) if owns_full else slice(self.lo, self.hi)
        full = flat_of(state["model_state"])
        self.master.copy_(full[sl])
        self.m.copy_(flat_of(state["optimizer_state"]["m"])[sl])
        self.v.copy_(flat_of(state["optimizer_state"]["v"])[sl])
        self.step = int(state["step"])
        self.micro_step = 0
        self.acc_grad.zero_()
        self.reduced.zero_()
        self._scatter_params(full)
        bufs = dict(self.model.named_buffers())
        for n, t in state.get("buffers", {}).items():
            if n not in bufs:
                raise ValueError(f"checkpoint buffer {n} is not in the model")
            bufs[n].copy_(t.to(bufs[n].device, bufs[n].dtype))


class DistributedTrainStepExecutor:
    """Executor seam (reference: src/flare/training/execution/executor.py:164-277).

    Wraps an engine and speaks in OptimizerUpdateWindow terms: ``micro_step``
    returns the result and the window, ``apply_update`` validates the window
    and applies the macro update when it should.
    """

    executor_kind = "distributed"

    def __init__(self, engine: TrainEngine):
        self.engine = engine
        self.plan = engine.plan
        self.executor_kind = f"zero{int(engine.stage)}"
        self._optimizer_step: int | None = None

    def prepare_execution(self, inputs: Any, targets: Any) -> None:
        del inputs, targets

    def micro_step(self, inputs: Any, targets: Any) -> tuple[TrainStepResult, OptimizerUpdateWindow]:
        result = self.engine.micro_step_once(inputs, targets)
        self._optimizer_step = result.step
        window = OptimizerUpdateWindow(
            micro_step=result.micro_step if result.micro_step > 0 else self.engine.micro_steps,
            accumulation_steps=self.plan.accumulation.micro_steps,
            at_boundary=result.optimizer_applied,
            should_apply_update=result.optimizer_applied and self.plan.update.apply_optimizer_at_boundary,
            optimizer_step=result.step)
        return result, window

    def apply_update(self, window: OptimizerUpdateWindow) -> bool:
        if self._optimizer_step is None:
            raise RuntimeError("optimizer update window requires a preceding micro-step")
        if window.optimizer_step != self._optimizer_step:
            raise ValueError(f"optimizer step mismatch: actual={window.optimizer_step}, expected={self._optimizer_step}")
        # the engine applies the update at the boundary inside micro_step; this
        # reports whether the window asked for it
        return bool(window.should_apply_update)

    def current_micro_step(self) -> int:
        return int(self.engine.micro_step)

    def finalize_checkpoint_window(self) -> bool:
        return self.engine.finalize_checkpoint_window()

    def capture_checkpoint_state(self) -> Mapping[str, Any]:
        return self.engine.capture_checkpoint_state()

    def checkpoint_layout(self) -> Mapping[str, Any]:
        return self.engine.checkpoint_layout()

    def restore_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        self.engine.restore_checkpoint_state(state)
        self._optimizer_step = int(state["step"])


ReplicatedTrainStepExecutor = DistributedTrainStepExecutor

__all__ = ["DistributedTrainStepExecutor", "ReplicatedTrainStepExecutor", "TrainEngine", "TrainStepResult"]
