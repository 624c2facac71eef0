"""Flat dense parameter storage and the dense optimizer step.

All dense parameters of a model live in four flat buffers:

* ``master``  fp32 master weights (the optimizer's copy),
* ``compute`` bf16 compute copy read by the GEMM / head kernels,
* ``grad``    fp32 gradients written by GEMM epilogues and reduction kernels,
* ``m``/``v`` optimizer moments.

Each parameter is a view at an offset aligned to 64 elements (128-byte aligned
bf16 views satisfy TMA's 16-byte rule).  With data parallelism the ``grad``
and ``compute`` buffers live in symmetric memory and the fused kernel
``adam_dp_fused`` performs reduce-scatter -> optimizer on the local shard ->
all-gather over NVLink in one launch (ZeRO-1: master and moments are sharded,
src/flare/training/zero/contracts.py:40-48; capability rules of
src/flare/jax/training/optimizers/base.py:70-150: elementwise optimizers
only, no global-norm clipping in sharded mode).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .._native import PEER_TIMEOUT_NS, DeviceStatus, native
from ..parallel.symm import FlagRegion, SymmetricHeap

ALIGN = 64
DENSE_OPT_KINDS = {"adam": 0, "adamw": 0, "sgd": 1, "adagrad": 2, "rmsprop": 3}


@dataclass(frozen=True)
class DenseOptimizerConfig:
    """Dense optimizer (reference factories: src/flare/jax/training/optimizers/optax_factories.py:14-149)."""

    kind: str = "adam"
    learning_rate: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.0
    momentum: float = 0.0
    nesterov: bool = False
    global_norm_clip: float | None = None

    def __post_init__(self):
        if self.kind not in DENSE_OPT_KINDS:
            raise ValueError(f"unsupported dense optimizer {self.kind!r}")

    @property
    def shardable(self) -> bool:
        """Elementwise update without a global reduction (sharded-update capability)."""
        return self.global_norm_clip is None

    def kernel_params(self, step: int) -> dict:
        t = max(int(step), 1)
        beta1 = self.momentum if self.kind == "sgd" else self.beta1
        beta2 = 0.9 if self.kind == "rmsprop" and self.beta2 == 0.999 else self.beta2
        return dict(kind=DENSE_OPT_KINDS[self.kind], lr=float(self.learning_rate), beta1=float(beta1),
                    beta2=float(beta2), eps=float(self.eps), weight_decay=float(self.weight_decay),
                    decoupled=1 if self.kind == "adamw" else 0, nesterov=1 if self.nesterov else 0,
                    bias_corr1=1.0 - math.pow(self.beta1, t), bias_corr2=1.0 - math.pow(beta2, t))


@dataclass
class ParamEntry:
    name: str
    shape: tuple[int, ...]
    offset: int
    numel: int
    init: str = "zeros"
    init_scale: float = 0.0
    zero_cols_from: int | None = None  # columns >= this start (and stay) zero: input padding
    zero_ranges: tuple[tuple[int, int], ...] = ()  # flat [lo, hi) ranges that start at zero (padding)


@dataclass
class FlatParams:
    """Registry of dense parameters and their flat storage."""

    entries: dict[str, ParamEntry] = field(default_factory=dict)
    size: int = 0

    def register(self, name: str, shape, init: str = "zeros", init_scale: float = 0.0,
                 zero_cols_from: int | None = None, zero_ranges: tuple[tuple[int, int], ...] = ()) -> ParamEntry:
        if name in self.entries:
            raise ValueError(f"duplicate parameter {name}")
        numel = 1
        for s in shape:
            numel *= int(s)
        off = (self.size + ALIGN - 1) // ALIGN * ALIGN
        e = ParamEntry(name, tuple(int(s) for s in shape), off, numel, init, init_scale, zero_cols_from,
                       tuple(zero_ranges))
        self.entries[name] = e
        self.size = off + numel
        return e

    def padded_size(self, world_size: int) -> int:
        q = ALIGN * max(world_size, 1)
        return (self.size + q - 1) // q * q


class DenseState:
    """Materialised flat buffers + optimizer for one rank."""

    def __init__(self, params: FlatParams, opt: DenseOptimizerConfig, *, device: torch.device,
                 rank: int = 0, world_size: int = 1, heap: SymmetricHeap | None = None, seed: int = 0,
                 timeout_ns: int = PEER_TIMEOUT_NS):
        if world_size > 1 and not opt.shardable:
            raise ValueError("sharded (ZeRO-1) dense update requires an optimizer without global-norm clipping")
        self.params, self.opt = params, opt
        self.device, self.rank, self.world = device, rank, world_size
        self.n = params.padded_size(world_size)
        self.step = 0
        self.timeout_ns = timeout_ns
        full_master = self._initial_values(seed)
        if world_size > 1:
            if heap is None:
                raise ValueError("a SymmetricHeap is required for world_size > 1")
            self._grad_buf = heap.alloc((self.n,), torch.float32)
            self._compute_buf = heap.alloc((self.n,), torch.bfloat16)
            self.grad = self._grad_buf.local
            self.compute = self._compute_buf.local
            self.grad.zero_()
            shard = self.n // world_size
            self.lo, self.hi = rank * shard, (rank + 1) * shard
            self.master = full_master[self.lo:self.hi].to(device).contiguous()
            self.m = torch.zeros(shard, dtype=torch.float32, device=device)
            self.v = torch.zeros(shard, dtype=torch.float32, device=device)
            self.flags = FlagRegion(heap, 2)
            self.peer_grad = self._grad_buf.peer_ptr_tensor(device)
            self.peer_compute = self._compute_buf.peer_ptr_tensor(device)
            self.compute.copy_(full_master.to(device).to(torch.bfloat16))
        else:
            self.lo, self.hi = 0, self.n
            self.master = full_master.to(device)
            self.grad = torch.zeros(self.n, dtype=torch.float32, device=device)
            self.compute = self.master.to(torch.bfloat16)
            self.m = torch.zeros(self.n, dtype=torch.float32, device=device)
            self.v = torch.zeros(self.n, dtype=torch.float32, device=device)
        self.status = DeviceStatus(device) if device.type == "cuda" else None
        # device-resident step counter: the optimizer kernels derive bias
        # corrections from it, so a captured CUDA graph stays correct on replay
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=device)

    def _initial_values(self, seed: int) -> torch.Tensor:
        g = torch.Generator().manual_seed(seed)
        flat = torch.zeros(self.n, dtype=torch.float32)
        for e in self.params.entries.values():
            if e.init == "zeros":
                continue
            if e.init == "ones":
                vals = torch.ones(e.numel)
            elif e.init == "uniform":
                vals = (torch.rand(e.numel, generator=g) * 2 - 1) * e.init_scale
            elif e.init == "normal":
                vals = torch.randn(e.numel, generator=g) * e.init_scale
            else:
                raise ValueError(f"unknown init {e.init!r}")
            if e.zero_cols_from is not None:
                vals = vals.view(e.shape).clone()
                vals[:, e.zero_cols_from:] = 0
                vals = vals.reshape(-1)
            for lo, hi in e.zero_ranges:
                vals[lo:hi] = 0
            flat[e.offset:e.offset + e.numel] = vals
        return flat

    # ---------------------------------------------------------------- views
    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        e = self.params.entries[name]
        return buf[e.offset:e.offset + e.numel].view(e.shape)

    def compute_view(self, name: str) -> torch.Tensor:
        return self._view(self.compute, name)

    def grad_view(self, name: str) -> torch.Tensor:
        return self._view(self.grad, name)

    def master_view(self, name: str) -> torch.Tensor:
        if self.world > 1:
            raise RuntimeError("master weights are sharded; use gather_master()")
        return self._view(self.master, name)

    # ------------------------------------------------------------ optimizer
    def apply(self, grad_scale: float = 1.0) -> None:
        """One optimizer step on the accumulated gradients; gradients are zeroed."""
        self.step += 1
        op = self.opt.kernel_params(self.step)
        if self.device.type != "cuda":
            self.step_dev += 1
            self._apply_reference(op, grad_scale)
            return
        native().increment_counter(self.step_dev.data_ptr())
        op["step_ptr"] = self.step_dev.data_ptr()
        if self.world > 1:
            native().adam_dp_fused(dict(
                world=self.world, rank=self.rank, lo=self.lo, hi=self.hi, peer_grad=self.peer_grad.data_ptr(),
                peer_param=self.peer_compute.data_ptr(), master_shard=self.master.data_ptr(),
                m_shard=self.m.data_ptr(), v_shard=self.v.data_ptr(), grad_scale=float(grad_scale), opt=op,
                flags_local=self.flags.local_ptr, peer_flags=self.flags.peer_ptrs.data_ptr(),
                flag_in=self.flags.slots(0), flag_out=self.flags.slots(1), epoch_ctr=self.flags.epoch_ptr(0),
                block_counter=self.flags.block_counter_ptr(0), status=self.status.ptr,
                timeout_ns=self.timeout_ns))
        else:
            native().adam_flat(dict(master=self.master.data_ptr(), grad=self.grad.data_ptr(), m=self.m.data_ptr(),
                                    v=self.v.data_ptr(), compute_copy=self.compute.data_ptr(), n=self.n,
                                    grad_scale=float(grad_scale), zero_grad=1, opt=op))

    def _apply_reference(self, op: dict, grad_scale: float) -> None:
        adam_reference(self.master, self.grad * grad_scale, self.m, self.v, op)
        self.compute.copy_(self.master.to(self.compute.dtype))
        self.grad.zero_()

    def gather_master(self) -> torch.Tensor:
        """Full fp32 master vector on this rank (all-gather over ranks when sharded)."""
        if self.world == 1:
            return self.master.clone()
        import torch.distributed as dist

        parts = [torch.empty_like(self.master) for _ in range(self.world)]
        dist.all_gather(parts, self.master)
        return torch.cat(parts)

    def state_dict(self) -> dict:
        return {"step": self.step, "master": self.gather_master().cpu(), "m": self._gather(self.m).cpu(),
                "v": self._gather(self.v).cpu()}

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t.clone()
        import torch.distributed as dist

        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t)
        return torch.cat(parts)

    def load_state_dict(self, state: dict) -> None:
        master = state["master"].to(self.device, torch.float32)
        if master.numel() != self.n:
            raise ValueError("checkpoint flat size does not match this model")
        self.step = int(state["step"])
        self.step_dev.fill_(self.step)
        self.master.copy_(master[self.lo:self.hi])
        self.m.copy_(state["m"].to(self.device)[self.lo:self.hi])
        self.v.copy_(state["v"].to(self.device)[self.lo:self.hi])
        self.compute.copy_(master.to(torch.bfloat16) if self.compute.dtype == torch.bfloat16 else master)
        self.grad.zero_()


def adam_reference(w: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor, op: dict) -> None:
    """fp32 reference of the fused dense optimizer kernel (in place)."""
    g = g.clone()
    if op["weight_decay"]:
        if op["decoupled"]:
            w -= op["lr"] * op["weight_decay"] * w
        else:
            g += op["weight_decay"] * w
    k = op["kind"]
    if k == 1:
        if op["beta1"]:
            m.mul_(op["beta1"]).add_(g)
            g = g + op["beta1"] * m if op["nesterov"] else m.clone()
        w -= op["lr"] * g
    elif k == 2:
        m += g * g
        w -= op["lr"] * g / (torch.sqrt(m) + op["eps"])
    elif k == 3:
        v.mul_(op["beta2"]).add_((1 - op["beta2"]) * g * g)
        w -= op["lr"] * g / (torch.sqrt(v) + op["eps"])
    else:
        m.mul_(op["beta1"]).add_((1 - op["beta1"]) * g)
        v.mul_(op["beta2"]).add_((1 - op["beta2"]) * g * g)
        w -= op["lr"] * (m / op["bias_corr1"]) / (torch.sqrt(v / op["bias_corr2"]) + op["eps"])


__all__ = ["DENSE_OPT_KINDS", "DenseOptimizerConfig", "DenseState", "FlatParams", "ParamEntry", "adam_reference"]
