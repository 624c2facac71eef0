"""Named-axis rank meshes and the sharding strategies built on them.

``ParallelMesh`` lays the ranks of a job out on named axes (row-major: the
last axis varies fastest, so ``ParallelMesh.from_axes(fsdp=4, tp=2)`` puts
the two ranks of a TP pair next to each other, the layout of
``DeviceMesh2D``).  A ``ShardSpec`` says, per tensor dimension, which mesh
axes split it (``None`` = not split); ``local_slice`` / ``shard`` give a
rank's contiguous block and ``assemble`` puts the blocks back.  Groups are
plain rank lists (what the fused kernels index peers with);
``torch_group(axis, rank)`` builds the matching process group for library
collectives.

Strategies (the reference's contracts in torch terms):

* ``DataParallelStrategy`` -- batch split over one axis, everything else
  replicated.
* ``ZeroShardingStrategy`` -- parameter / optimizer-state / gradient specs
  per ZeRO stage, from the stage table of ``training.contracts``; the specs
  of a flattened state and the per-rank blocks of a state dict.
* ``CheckpointShardingStrategy`` -- a saved tensor is split on its first
  dimension divisible by the axis size, else replicated.

Reference: ``ParallelMesh`` (src/flare/jax/mesh.py:131) and the strategies of
src/flare/jax/training/strategy.py:33,54,152.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch

from ..training.contracts import ZeroPartitionContract, ZeroStage, zero_partition_contract


@dataclass(frozen=True)
class ShardSpec:
    """Per tensor dimension: the mesh axes splitting it (a name, a tuple of names, or None)."""

    dims: tuple[Any, ...] = ()

    @property
    def is_replicated(self) -> bool:
        return all(d is None for d in self.dims)

    def axes_of(self, dim: int) -> tuple[str, ...]:
        if dim >= len(self.dims) or self.dims[dim] is None:
            return ()
        d = self.dims[dim]
        return (d,) if isinstance(d, str) else tuple(d)


@dataclass(frozen=True)
class ParallelMesh:
    axis_names: tuple[str, ...]
    shape: tuple[int, ...]

    def __post_init__(self):
        if not self.axis_names:
            raise ValueError("axis_names must be non-empty")
        if len(set(self.axis_names)) != len(self.axis_names):
            raise ValueError(f"axis_names must be unique, got {self.axis_names}")
        if len(self.shape) != len(self.axis_names):
            raise ValueError("one size per axis")
        for n, s in zip(self.axis_names, self.shape):
            if not isinstance(n, str) or not n:
                raise ValueError("axis name must be non-empty")
            if isinstance(s, bool) or not isinstance(s, int) or s <= 0:
                raise ValueError(f"axis {n!r} size must be positive, got {s}")

    # ------------------------------------------------------------ builders
    @classmethod
    def from_axes(cls, *, world_size: int | None = None, **axes: int) -> "ParallelMesh":
        if not axes:
            raise ValueError("at least one axis must be specified")
        mesh = cls(tuple(axes), tuple(axes.values()))
        if world_size is not None and mesh.size != world_size:
            raise ValueError(f"world size {world_size} does not match axes product {mesh.size} (axes={axes})")
        return mesh

    @classmethod
    def from_dp(cls, world_size: int, axis_name: str = "data") -> "ParallelMesh":
        return cls.from_axes(**{axis_name: int(world_size)})

    # ------------------------------------------------------------ geometry
    @property
    def size(self) -> int:
        return math.prod(self.shape)

    def axis_size(self, name: str) -> int:
        return self.shape[self._axis(name)]

    def _axis(self, name: str) -> int:
        try:
            return self.axis_names.index(name)
        except ValueError:
            raise ValueError(f"axis {name!r} is not present in mesh axes {self.axis_names}") from None

    def coords(self, rank: int) -> dict[str, int]:
        if not 0 <= rank < self.size:
            raise ValueError(f"rank {rank} outside the mesh of {self.size}")
        out, r = {}, rank
        for n, s in zip(reversed(self.axis_names), reversed(self.shape)):
            out[n] = r % s
            r //= s
        return {n: out[n] for n in self.axis_names}

    def rank_of(self, **coords: int) -> int:
        r = 0
        for n, s in zip(self.axis_names, self.shape):
            c = coords.get(n, 0)
            if not 0 <= c < s:
                raise ValueError(f"coordinate {n}={c} outside [0, {s})")
            r = r * s + c
        return r

    def group(self, axis: str | tuple[str, ...], rank: int) -> list[int]:
        """Ranks that differ from ``rank`` only along ``axis`` (or several axes), in axis order."""
        names = (axis,) if isinstance(axis, str) else tuple(axis)
        for n in names:
            self._axis(n)
        base = self.coords(rank)
        out = [base]
        for n in names:
            out = [dict(c, **{n: i}) for c in out for i in range(self.axis_size(n))]
        return sorted(self.rank_of(**c) for c in out)

    def groups(self, axis: str | tuple[str, ...]) -> list[list[int]]:
        seen, out = set(), []
        for r in range(self.size):
            g = tuple(self.group(axis, r))
            if g not in seen:
                seen.add(g)
                out.append(list(g))
        return out

    def torch_group(self, axis: str | tuple[str, ...], rank: int):
        """The process group of ``rank``'s ``axis`` group (every rank must call this for every group)."""
        import torch.distributed as dist

        mine = None
        for g in self.groups(axis):
            pg = dist.new_group(g)
            if rank in g:
                mine = pg
        return mine

    # ------------------------------------------------------------ specs
    @property
    def replicated(self) -> ShardSpec:
        return ShardSpec(())

    def named(self, *dims: Any) -> ShardSpec:
        for d in dims:
            for n in ((d,) if isinstance(d, str) else (d or ())):
                self._axis(n)
        return ShardSpec(tuple(dims))

    def local_slice(self, spec: ShardSpec, shape: tuple[int, ...], rank: int) -> tuple[slice, ...]:
        """``rank``'s block of a tensor of ``shape`` under ``spec`` (each split dim divided evenly)."""
        c = self.coords(rank)
        out = []
        for dim, n in enumerate(shape):
            axes = spec.axes_of(dim)
            parts = math.prod(self.axis_size(a) for a in axes) if axes else 1
            if n % parts:
                raise ValueError(f"dim {dim} of size {n} does not divide into {parts} shards")
            idx = 0
            for a in axes:
                idx = idx * self.axis_size(a) + c[a]
            step = n // parts
            out.append(slice(idx * step, (idx + 1) * step))
        return tuple(out)

    def shard(self, tensor: torch.Tensor, spec: ShardSpec, rank: int) -> torch.Tensor:
        return tensor[self.local_slice(spec, tuple(tensor.shape), rank)]

    def assemble(self, shards: Mapping[int, torch.Tensor], spec: ShardSpec, shape: tuple[int, ...]) -> torch.Tensor:
        """The full tensor from every rank's block (replicated dims: any rank's copy)."""
        first = next(iter(shards.values()))
        out = torch.empty(shape, dtype=first.dtype, device=first.device)
        covered = torch.zeros(shape, dtype=torch.bool) if math.prod(shape) <= (1 << 24) else None
        for r, t in shards.items():
            sl = self.local_slice(spec, shape, r)
            out[sl] = t
            if covered is not None:
                covered[sl] = True
        if covered is not None and not bool(covered.all()):
            raise ValueError("the shards do not cover the tensor")
        return out


class DataParallelStrategy:
    def __init__(self, mesh: ParallelMesh, axis_name: str = "data"):
        mesh._axis(axis_name)
        self.mesh, self.axis_name = mesh, axis_name

    def batch_sharding(self, *extra_dims: Any) -> ShardSpec:
        return self.mesh.named(self.axis_name, *extra_dims)

    @property
    def replicated(self) -> ShardSpec:
        return self.mesh.replicated


class ZeroShardingStrategy:
    """Parameter / optimizer / gradient partitions of a ZeRO stage over one mesh axis.

    A sharded partition splits the (flattened, padded) state along dim 0 over the axis, which is the
    layout of ``training.flat.FlatParams`` shards and of the fused ZeRO kernels."""

    def __init__(self, mesh: ParallelMesh, stage: ZeroStage, axis_name: str = "fsdp"):
        mesh._axis(axis_name)
        if not isinstance(stage, ZeroStage):
            raise TypeError(f"stage must be ZeroStage, got {type(stage).__name__}")
        self.mesh, self.stage, self.axis_name = mesh, stage, axis_name

    @classmethod
    def from_execution_plan(cls, plan, mesh: ParallelMesh) -> "ZeroShardingStrategy":
        from ..training.contracts import TrainingExecutionPlan

        if not isinstance(plan, TrainingExecutionPlan):
            raise TypeError(f"plan must be TrainingExecutionPlan, got {type(plan).__name__}")
        return cls(mesh, plan.zero.stage, plan.zero.axis_name)

    def zero_contract(self) -> ZeroPartitionContract:
        return zero_partition_contract(self.stage, axis_name=self.axis_name)

    def _spec(self, partition: str) -> ShardSpec:
        if partition == "replicated":
            return self.mesh.replicated
        if partition == "sharded":
            return self.mesh.named(self.axis_name)
        raise ValueError(f"unknown partition type {partition!r}")

    def zero_parameter_sharding(self) -> ShardSpec:
        return self._spec(self.zero_contract().parameter_partition)

    def zero_optimizer_sharding(self) -> ShardSpec:
        return self._spec(self.zero_contract().optimizer_state_partition)

    def zero_gradient_sharding(self) -> ShardSpec:
        return self._spec(self.zero_contract().gradient_partition)

    def zero_state_specs(self, model_leaf_count: int, total_leaf_count: int) -> tuple[ShardSpec, ...]:
        if model_leaf_count < 0 or total_leaf_count < 0 or model_leaf_count > total_leaf_count:
            raise ValueError(f"invalid leaf counts: model={model_leaf_count}, total={total_leaf_count}")
        m, o = self.zero_parameter_sharding(), self.zero_optimizer_sharding()
        return tuple(m if i < model_leaf_count else o for i in range(total_leaf_count))

    def zero_gradient_specs(self, leaf_count: int) -> tuple[ShardSpec, ...]:
        if leaf_count < 0:
            raise ValueError(f"leaf_count must be non-negative, got {leaf_count}")
        return (self.zero_gradient_sharding(),) * leaf_count

    def padded_numel(self, numel: int) -> int:
        """Flattened size padded to a multiple of the axis size (every shard equal)."""
        k = self.mesh.axis_size(self.axis_name)
        return -(-int(numel) // k) * k

    def shard_flat(self, flat: torch.Tensor, partition: str, rank: int) -> torch.Tensor:
        """``rank``'s block of a flattened state vector under a partition kind."""
        if partition == "replicated":
            return flat
        n = self.padded_numel(flat.numel())
        if n != flat.numel():
            flat = torch.cat([flat, flat.new_zeros(n - flat.numel())])
        return self.mesh.shard(flat, self._spec(partition), rank)

    def shard_model(self, module: torch.nn.Module, rank: int) -> dict[str, torch.Tensor]:
        """This rank's blocks of the module's flattened parameters (all of them when replicated)."""
        part = self.zero_contract().parameter_partition
        return {n: self.shard_flat(p.detach().reshape(-1), part, rank) for n, p in module.named_parameters()}

    def shard_optimizer(self, optimizer_state: Mapping[str, torch.Tensor], rank: int) -> dict[str, torch.Tensor]:
        part = self.zero_contract().optimizer_state_partition
        return {k: self.shard_flat(v.reshape(-1), part, rank) for k, v in optimizer_state.items()}


class CheckpointShardingStrategy:
    """Saved tensors split on their first dimension divisible by the axis size (else replicated)."""

    def __init__(self, mesh: ParallelMesh, axis_name: str):
        mesh._axis(axis_name)
        self.mesh, self.axis_name = mesh, axis_name

    def checkpoint_sharding(self, shape: tuple[int, ...]) -> ShardSpec:
        k = self.mesh.axis_size(self.axis_name)
        if k > 1:
            for dim, n in enumerate(shape):
                if n > 0 and n % k == 0:
                    return self.mesh.named(*([None] * dim), self.axis_name)
        return self.mesh.replicated

    def local_shards(self, state: Mapping[str, torch.Tensor], rank: int) -> dict[str, torch.Tensor]:
        """What ``rank`` writes: its block of every tensor (replicated tensors only on axis index 0)."""
        first = self.mesh.coords(rank)[self.axis_name] == 0
        out = {}
        for k, t in state.items():
            spec = self.checkpoint_sharding(tuple(t.shape))
            if spec.is_replicated:
                if first:
                    out[k] = t
            else:
                out[k] = self.mesh.shard(t, spec, rank)
        return out

    def assemble(self, per_rank: Mapping[int, Mapping[str, torch.Tensor]],
                 shapes: Mapping[str, tuple[int, ...]]) -> dict[str, torch.Tensor]:
        out = {}
        for k, shape in shapes.items():
            spec = self.checkpoint_sharding(tuple(shape))
            holders = {r: st[k] for r, st in per_rank.items() if k in st}
            if not holders:
                raise KeyError(f"no rank saved {k!r}")
            out[k] = next(iter(holders.values())) if spec.is_replicated else self.mesh.assemble(holders, spec, shape)
        return out


__all__ = ["CheckpointShardingStrategy", "DataParallelStrategy", "ParallelMesh", "ShardSpec",
           "ZeroShardingStrategy"]
