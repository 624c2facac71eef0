"""Fused dense optimizer for any ``nn.Module``: flat buffers, tcgen05 gradients, no NCCL.

``FusedDenseParameters(module, opt, ...)`` moves every parameter of an
arbitrary module into one flat layout (the layout of
``flare_b200.training.flat``) and binds the module to it:

* each parameter's data becomes a bf16 view of the flat *compute* buffer, so
  the module computes in bf16 from weights the fused optimizer refreshes in
  place after every step;
* each parameter carries ``_flare_grad``, an fp32 view of the flat gradient
  buffer.  ``TcLinear`` layers (the library's MLP, gates, experts) write
  ``dW`` and ``db`` straight into it from the tcgen05 GEMM epilogues
  (accumulating, so micro-steps add up); any other parameter's autograd
  gradient is added into it by a post-accumulate hook;
* ``step()`` runs one fused update: at one GPU the flat Adam kernel, at N
  GPUs the fused reduce-scatter + Adam + all-gather over NVLink peer memory
  (ZeRO-1, ``adam_dp_fused``); gradients come back zeroed.

So a user model trains on the same fused kernels as the hand-written
towers, with gradients and parameters that never pass through NCCL.
Reference: the flat-state engine and sharded optimizer update of
src/flare/jax/training/engines/distributed.py:187-1301 and
src/flare/jax/training/state/layout.py:12-105.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .flat import DenseOptimizerConfig, DenseState, FlatParams


class FusedDenseParameters:
    def __init__(self, module: nn.Module, opt: DenseOptimizerConfig, *, device: torch.device, rank: int = 0,
                 world_size: int = 1, heap=None, broadcast_from_rank0: bool = True):
        self.module = module
        self.names: list[str] = []
        params = FlatParams()
        self._params: list[nn.Parameter] = []
        for name, p in _stack_grouped(module.named_parameters()):
            if not p.requires_grad:
                continue
            params.register(name, tuple(p.shape))
            self.names.append(name)
            self._params.append(p)
        if not self._params:
            raise ValueError("the module has no trainable parameters")
        self.state = DenseState(params, opt, device=device, rank=rank, world_size=world_size, heap=heap)
        init = torch.zeros(self.state.n, dtype=torch.float32, device=device)
        for name, p in zip(self.names, self._params):
            e = params.entries[name]
            init[e.offset:e.offset + e.numel] = p.detach().to(device, torch.float32).reshape(-1)
        if world_size > 1 and broadcast_from_rank0:
            import torch.distributed as dist

            dist.broadcast(init, 0)  # set-up only: every rank starts from rank 0's weights
        self.state.master.copy_(init[self.state.lo:self.state.hi])
        self.state.compute.copy_(init.to(self.state.compute.dtype))
        self._hooks = []
        for name, p in zip(self.names, self._params):
            p.data = self.state.compute_view(name)
            p._flare_grad = self.state.grad_view(name)  # written by TcLinear, or by the hook below
            self._hooks.append(p.register_post_accumulate_grad_hook(_accumulate_into_flat))

    @property
    def grad(self) -> torch.Tensor:
        return self.state.grad

    def step(self, grad_scale: float = 1.0) -> None:
        """One fused optimizer step on the accumulated flat gradients (which it zeroes)."""
        self.state.apply(grad_scale)

    def master_values(self) -> dict[str, torch.Tensor]:
        """fp32 master weights by parameter name (gathered over ranks)."""
        full = self.state.gather_master()
        out = {}
        for name in self.names:
            e = self.state.params.entries[name]
            out[name] = full[e.offset:e.offset + e.numel].view(e.shape)
        return out

    def state_dict(self) -> dict:
        return {"names": list(self.names), **self.state.state_dict()}

    def load_state_dict(self, st: dict) -> None:
        if list(st.get("names", self.names)) != self.names:
            raise ValueError("checkpoint parameters do not match this module")
        self.state.load_state_dict(st)


def _stack_grouped(named):
    """Parameters in module order, except that the members of a stack group (``p._flare_stack = (group,
    kind, index)``, set by layers that run several equal-shaped parameters as one GEMM operand) are
    registered back to back, in index order, where the group's first member appears."""
    named = list(named)
    groups: dict = {}
    for n, p in named:
        key = getattr(p, "_flare_stack", None)
        if key is not None:
            groups.setdefault(key[:2], []).append((key[2], n, p))
    out, done = [], set()
    for n, p in named:
        key = getattr(p, "_flare_stack", None)
        if key is None:
            out.append((n, p))
        elif key[:2] not in done:
            done.add(key[:2])
            out.extend((m, q) for _, m, q in sorted(groups[key[:2]], key=lambda t: t[0]))
    return out


def _accumulate_into_flat(p: torch.Tensor) -> None:
    """Autograd gradient of a parameter that no fused layer writes: add it to the flat buffer."""
    if p.grad is not None:
        p._flare_grad.add_(p.grad.to(torch.float32))
        p.grad = None


__all__ = ["FusedDenseParameters"]
