"""Device meshes for one node: named axes, rank groups, sparse partition mapping.

``DeviceMesh2D(tp, fsdp)`` lays ``world = tp * fsdp`` ranks out with the
tensor-parallel axis innermost (``rank = d * tp + t``), so the two ranks of a
TP pair are neighbours.  Groups are plain rank lists; the fused kernels use
them to index peers in symmetric memory (no communicator objects needed), and
``torch_groups()`` builds the matching ``torch.distributed`` groups for the
library baseline.

``SparsePartitionMapping`` keeps the sparse-table partitioning independent of
the dense mesh, as the reference does (src/flare/mesh/mapping.py:11): tables
are sharded over every rank of the node whatever the dense layout is.
The reference's mesh constructors are src/flare/mesh/topology.py:20-35 and its
named-axis mesh is ``ParallelMesh`` (src/flare/jax/training/sharding/mesh.py).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class DeviceMesh2D:
    tp: int
    fsdp: int

    def __post_init__(self):
        if self.tp < 1 or self.fsdp < 1:
            raise ValueError("mesh axes must be >= 1")

    @property
    def world(self) -> int:
        return self.tp * self.fsdp

    @classmethod
    def for_world(cls, world: int, tp: int = 2) -> "DeviceMesh2D":
        tp = min(tp, world)
        if world % tp:
            raise ValueError(f"world size {world} is not divisible by tp={tp}")
        return cls(tp, world // tp)

    def coords(self, rank: int) -> tuple[int, int]:
        """(tp index, fsdp index) of a rank."""
        if not 0 <= rank < self.world:
            raise ValueError("rank outside the mesh")
        return rank % self.tp, rank // self.tp

    def tp_group(self, rank: int) -> list[int]:
        _, d = self.coords(rank)
        return [d * self.tp + t for t in range(self.tp)]

    def fsdp_group(self, rank: int) -> list[int]:
        t, _ = self.coords(rank)
        return [d * self.tp + t for d in range(self.fsdp)]

    def world_group(self) -> list[int]:
        return list(range(self.world))

    def torch_groups(self):
        """(tp groups, fsdp groups) as torch.distributed groups; every rank must call this."""
        import torch.distributed as dist

        tp = {}
        for d in range(self.fsdp):
            ranks = [d * self.tp + t for t in range(self.tp)]
            tp[tuple(ranks)] = dist.new_group(ranks)
        fs = {}
        for t in range(self.tp):
            ranks = [d * self.tp + t for d in range(self.fsdp)]
            fs[tuple(ranks)] = dist.new_group(ranks)
        return tp, fs


@dataclass(frozen=True)
class SparsePartitionMapping:
    """Sparse axes (where tables are partitioned) vs replica axes (where they are not)."""

    sparse_ranks: tuple[int, ...]
    replica_groups: tuple[tuple[int, ...], ...] = ()

    @classmethod
    def over_node(cls, world: int) -> "SparsePartitionMapping":
        return cls(tuple(range(world)), ())

    @property
    def num_partitions(self) -> int:
        return len(self.sparse_ranks)

    def partition_of(self, rank: int) -> int:
        return self.sparse_ranks.index(rank)


__all__ = ["DeviceMesh2D", "SparsePartitionMapping"]
