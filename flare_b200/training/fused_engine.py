"""The generic training engine's API on the fused B200 path.

``FusedTrainEngine`` runs any autograd model with the contract of
``training.engine.TrainEngine`` (``micro_step_once``, windows of
``plan.accumulation.micro_steps`` micro-steps with the update at the
boundary, ``apply_accumulated_update``, ``finalize_checkpoint_window``,
``input_gradients``, logical-shape checkpoints) but moves the dense state
into ``FusedDenseParameters``: the parameters compute in bf16 from the flat
compute buffer, every ``TcLinear`` writes its weight and bias gradients
straight into the flat fp32 gradient buffer (other parameters through a
gradient hook), gradients add up across the micro-steps of a window, and
one fused update applies them: the flat Adam kernel on one GPU, the fused
reduce-scatter + Adam + all-gather over NVLink peer memory on several
(ZeRO-1 placement; stages 0-2 have the same arithmetic and differ only in
where state lives, so they all map to it).  No NCCL call moves a gradient
or a parameter; the loss mean over ranks and float-buffer averaging are
scalar / small collectives.

``make_train_engine`` picks this engine on CUDA when the plan allows it
(ZeRO stage 0-2, global shard scope, boundary sync, an elementwise
optimizer) and the eager ``TrainEngine`` (the library baseline) otherwise.

Reference behaviour: the micro-step / macro-update engine of
src/flare/jax/training/engines/distributed.py:1017-1180.
"""
from __future__ import annotations

import hashlib
from collections.abc import Callable, Mapping
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from .contracts import TrainingExecutionPlan, ZeroStage
from .engine import TrainEngine, TrainStepResult
from .flat import DenseOptimizerConfig
from .fused_module import FusedDenseParameters


def fused_engine_supported(plan: TrainingExecutionPlan, optimizer: DenseOptimizerConfig, device: torch.device) -> bool:
    return (device.type == "cuda" and plan.zero.stage is not ZeroStage.PARAMETER
            and plan.zero.shard_scope == "global" and plan.accumulation.sync_mode == "boundary"
            and plan.update.apply_optimizer_at_boundary and optimizer.shardable)


class FusedTrainEngine:
    def __init__(self, model: nn.Module, loss_fn: Callable[[Any, Any], torch.Tensor], plan: TrainingExecutionPlan,
                 optimizer: DenseOptimizerConfig, *, device: torch.device | None = None,
                 forward: Callable[[nn.Module, Any], Any] | None = None, heap=None, sync_buffers: bool = True):
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        if not fused_engine_supported(plan, optimizer, self.device):
            raise ValueError("the fused engine needs CUDA, ZeRO stage 0-2 with global scope, boundary sync and an "
                             "elementwise optimizer")
        self.model, self.loss_fn, self.plan, self.opt = model, loss_fn, plan, optimizer
        self.forward_fn = forward or (lambda m, x: m(x))
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.stage = plan.zero.stage
        self.micro_steps = plan.accumulation.micro_steps
        self.micro_step = 0
        self.sync_buffers = sync_buffers
        model.to(self.device)
        if self.world > 1 and heap is None:
            from ..parallel.symm import SymmetricHeap

            n = sum(p.numel() for p in model.parameters() if p.requires_grad)
            heap = SymmetricHeap(6 * (n + 4096 * self.world) + (16 << 20), rank=self.rank, world_size=self.world,
                                 device=self.device)
        self.heap = heap
        self.dense = FusedDenseParameters(model, optimizer, device=self.device, rank=self.rank, world_size=self.world,
                                          heap=heap)
        self.names = list(self.dense.names)
        self.shapes = {n: tuple(p.shape) for n, p in model.named_parameters() if n in self.dense.names}
        self.last_loss: float | None = None

    @property
    def step(self) -> int:
        return self.dense.state.step

    def micro_step_once(self, inputs: Any, targets: Any) -> TrainStepResult:
        outputs = self.forward_fn(self.model, inputs)
        loss = self.loss_fn(outputs, targets)
        loss.backward()  # gradients add into the flat buffer (TcLinear epilogues and the gradient hooks)
        self._sync_buffer_state()
        self.micro_step += 1
        applied = False
        if self.micro_step == self.micro_steps:
            self.apply_accumulated_update()
            applied = True
        mean_loss = loss.detach().float()
        if self.world > 1:
            mean_loss = mean_loss.clone()
            dist.all_reduce(mean_loss)
            mean_loss = mean_loss / self.world
        self.last_loss = float(mean_loss)
        return TrainStepResult(mean_loss, self.micro_steps if applied else self.micro_step, self.step, applied, outputs)

    def _sync_buffer_state(self) -> None:
        if self.world == 1 or not self.sync_buffers:
            return
        for _, b in self.model.named_buffers():
            if b.is_floating_point():
                t = b.detach().float().clone()
                dist.all_reduce(t)
                b.copy_((t / self.world).to(b.dtype))

    def input_gradients(self, inputs: Mapping[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        from .gradients import input_gradients

        return input_gradients(inputs, world_size=self.world, micro_steps=self.micro_steps)

    def apply_accumulated_update(self, micro_steps: int | None = None) -> None:
        """One fused update on the window's summed gradients: mean over micro-steps and ranks."""
        n = micro_steps or self.micro_steps
        self.dense.step(grad_scale=1.0 / (n * self.world))
        self.micro_step = 0

    def finalize_checkpoint_window(self) -> bool:
        if self.micro_step == 0:
            return False
        self.apply_accumulated_update(self.micro_step)
        return True

    # ------------------------------------------------------------ checkpoints (TrainEngine format)
    def schema_digest(self) -> str:
        h = hashlib.sha256()
        for n in self.names:
            h.update(f"{n}:{self.shapes[n]}:float32;".encode())
        return h.hexdigest()

    def checkpoint_layout(self) -> Mapping[str, Any]:
        return {"leaves": [(n, self.shapes[n], "float32") for n in self.names], "schema_digest": self.schema_digest(),
                "zero_stage": int(self.stage), "world_size": self.world, "shard_scope": "global",
                "shards": self.world}

    def _unflatten(self, flat: torch.Tensor) -> dict[str, torch.Tensor]:
        out = {}
        for n in self.names:
            e = self.dense.state.params.entries[n]
            out[n] = flat[e.offset:e.offset + e.numel].view(self.shapes[n]).detach().cpu().clone()
        return out

    def capture_checkpoint_state(self) -> dict[str, Any]:
        if self.micro_step != 0:
            raise RuntimeError("checkpoint capture requires an optimizer-window boundary")
        st = self.dense.state.state_dict()
        return {"step": self.step, "schema_digest": self.schema_digest(),
                "model_state": self._unflatten(st["master"]),
                "optimizer_state": {"m": self._unflatten(st["m"]), "v": self._unflatten(st["v"])},
                "buffers": {n: b.detach().cpu().clone() for n, b in self.model.named_buffers()}}

    def restore_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        if state.get("schema_digest") not in (None, self.schema_digest()):
            raise ValueError("checkpoint schema does not match this model")
        st = self.dense.state.state_dict()
        flat = {k: torch.zeros_like(st[k]) for k in ("master", "m", "v")}
        for key, src in (("master", state["model_state"]), ("m", state["optimizer_state"]["m"]),
                         ("v", state["optimizer_state"]["v"])):
            for n in self.names:
                e = self.dense.state.params.entries[n]
                t = src[n]
                if tuple(t.shape) != self.shapes[n]:
                    raise ValueError(f"checkpoint leaf {n} has shape {tuple(t.shape)}, expected {self.shapes[n]}")
                flat[key][e.offset:e.offset + e.numel] = t.reshape(-1).float()
        self.dense.state.load_state_dict({**st, **flat, "step": int(state["step"])})
        self.micro_step = 0
        bufs = dict(self.model.named_buffers())
        for n, t in state.get("buffers", {}).items():
            if n not in bufs:
                raise ValueError(f"checkpoint buffer {n} is not in the model")
            bufs[n].copy_(t.to(bufs[n].device, bufs[n].dtype))


def make_train_engine(model: nn.Module, loss_fn, plan: TrainingExecutionPlan, optimizer: DenseOptimizerConfig, *,
                      device: torch.device | None = None, **kwargs):
    """The fused engine on CUDA when the plan allows it, the eager ``TrainEngine`` otherwise."""
    dev = device or next(model.parameters()).device
    if fused_engine_supported(plan, optimizer, dev):
        allowed = {k: v for k, v in kwargs.items() if k in ("forward", "heap", "sync_buffers")}
        return FusedTrainEngine(model, loss_fn, plan, optimizer, device=dev, **allowed)
    return TrainEngine(model, loss_fn, plan, optimizer, device=dev, **kwargs)


__all__ = ["FusedTrainEngine", "fused_engine_supported", "make_train_engine"]
