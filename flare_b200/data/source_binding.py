"""Binding a planned dataset source to the job's reader ranks.

``ScheduledDatasetSource`` describes a finite source (a ``SourceFactory``,
the global batch size, the completion policy and the assignment policy)
and derives from it what the readers of a job need:

* the **reader topology**: the execution cycle (for each step of the
  repeating schedule, the reader ranks active in it; every rank reads every
  step by default), which must activate the same number of readers in
  every step, and per reader rank its demand of ``global_batch /
  active_readers`` rows, optionally pinned to the node the rank runs on;
* the **tail layout**: what happens to the rows after the last full batch,
  from the completion policy (drop -> discard the remainder, carry -> keep
  it pending for the next source, require -> reject a remainder, pad ->
  synthesise padded rows with a validity mask);
* the **scan binding**: the planned work items, an identity of the plan
  (a digest of every item's ranges, checked again on restore), the initial
  cursor, the topology, the tail layout and the per-rank assignment
  (round-robin: item k to reader ``k % readers``, the dealing of
  ``BatchReader``; or contiguous blocks balanced by rows);
* read sessions (``create_session``) and per-rank ``BatchReader`` objects.

Reference behaviour: ``WorkItemScheduledDatasetSourceDescriptor``
(src/flare/runtime/fluxway/source.py:37; tail mapping :70-77, reader
topology :79-109, sessions :182-198).  The reference asks its runtime's
control plane for the execution cycle; here the job is one process per GPU
and the cycle is given (or every rank every step).
"""
from __future__ import annotations

import hashlib
import json
from collections.abc import Sequence
from dataclasses import dataclass, field
from enum import Enum
from typing import Any

from .reader import BatchReader
from .sources import CompletionPolicy, SourceFactory, WorkItem


class TailLayoutMode(str, Enum):
    DISCARD_REMAINDER = "discard_remainder"
    RETAIN_PENDING = "retain_pending"
    REJECT_REMAINDER = "reject_remainder"
    SYNTHESIZE_PADDING = "synthesize_padding"


_TAIL = {
    CompletionPolicy.DROP: TailLayoutMode.DISCARD_REMAINDER,
    CompletionPolicy.CARRY: TailLayoutMode.RETAIN_PENDING,
    CompletionPolicy.REQUIRE: TailLayoutMode.REJECT_REMAINDER,
    CompletionPolicy.PAD: TailLayoutMode.SYNTHESIZE_PADDING,
}


def tail_layout_mode(policy: str | CompletionPolicy) -> TailLayoutMode:
    return _TAIL[CompletionPolicy.from_value(policy)]


class AssignmentPolicy(str, Enum):
    ROUND_ROBIN = "round_robin"
    CONTIGUOUS = "contiguous"

    @classmethod
    def from_value(cls, value) -> "AssignmentPolicy":
        if isinstance(value, cls):
            return value
        try:
            return cls(str(value))
        except ValueError:
            raise ValueError(f"unknown assignment policy {value!r}; expected one of "
                             f"{[p.value for p in cls]}") from None


def reader_worker_id(job_id: str, operator: str, rank: int) -> str:
    return f"{job_id}/{operator}/{int(rank)}"


@dataclass(frozen=True)
class RankDemand:
    worker_id: str
    rows_per_step: int


@dataclass(frozen=True)
class ReaderGroup:
    worker_id: str
    demands: tuple[RankDemand, ...]
    node_id: str | None = None


@dataclass(frozen=True)
class ReaderTopology:
    global_cardinality: int
    groups: tuple[ReaderGroup, ...]
    execution_cycle: tuple[tuple[int, ...], ...]

    def rows_per_reader(self) -> int:
        return self.groups[0].demands[0].rows_per_step if self.groups else 0

    def active_readers(self, step: int) -> tuple[int, ...]:
        return self.execution_cycle[step % len(self.execution_cycle)]


@dataclass(frozen=True)
class SourceScanBinding:
    items: tuple[WorkItem, ...]
    identity: str
    initial_cursor: int
    topology: ReaderTopology
    tail_layout_mode: TailLayoutMode
    assignment_policy: AssignmentPolicy
    assignments: tuple[tuple[int, ...], ...]   # per reader rank: global work-item ids

    def check_identity(self, identity: str) -> None:
        """A restore must see the same plan it was saved from."""
        if identity != self.identity:
            raise ValueError("the source plan changed since the checkpoint (binding identity differs)")


def plan_identity(items: Sequence[WorkItem]) -> str:
    h = hashlib.sha256()
    for it in items:
        h.update(json.dumps([it.item_id, [[r.path, r.start, r.stop] for r in it.ranges]]).encode())
    return h.hexdigest()


@dataclass(frozen=True)
class ScheduledDatasetSource:
    source_factory: SourceFactory
    global_batch_size: int
    completion_policy: str | CompletionPolicy = "pad"
    assignment_policy: str | AssignmentPolicy = AssignmentPolicy.ROUND_ROBIN
    job_id: str = field(default="job", kw_only=True)
    operator: str = field(default="reader", kw_only=True)

    def __post_init__(self):
        if not callable(getattr(self.source_factory, "plan", None)) or \
                not callable(getattr(self.source_factory, "create_session", None)):
            raise TypeError("source descriptor requires a SourceFactory (plan / create_session)")
        if type(self.global_batch_size) is not int or self.global_batch_size <= 0:
            raise ValueError("dataset global_batch_size must be positive")
        CompletionPolicy.from_value(self.completion_policy)
        object.__setattr__(self, "assignment_policy", AssignmentPolicy.from_value(self.assignment_policy))

    # -------------------------------------------------------------- topology
    def build_reader_topology(self, world_size: int, *, cycle: Sequence[Sequence[int]] | None = None,
                              node_ids: Sequence[str] | None = None) -> ReaderTopology:
        if world_size < 1:
            raise ValueError("world_size must be >= 1")
        cyc = tuple(tuple(int(r) for r in step) for step in (cycle or [range(world_size)]))
        if not cyc or not cyc[0]:
            raise ValueError("the execution cycle needs at least one active reader")
        active = len(cyc[0])
        if any(len(step) != active for step in cyc):
            raise ValueError("dataset source requires uniform active reader counts")
        if any(not 0 <= r < world_size for step in cyc for r in step):
            raise ValueError("execution cycle names a rank outside the job")
        if node_ids is not None and len(node_ids) != world_size:
            raise ValueError("node_ids must contain one node id per reader rank")
        if self.global_batch_size % active:
            raise ValueError("global_batch_size must divide by the active reader count")
        per = self.global_batch_size // active
        groups = tuple(ReaderGroup(reader_worker_id(self.job_id, self.operator, r),
                                   (RankDemand(reader_worker_id(self.job_id, self.operator, r), per),),
                                   None if node_ids is None else str(node_ids[r]))
                       for r in range(world_size))
        return ReaderTopology(self.global_batch_size, groups, cyc)

    def tail_layout_mode(self) -> TailLayoutMode:
        return tail_layout_mode(self.completion_policy)

    # -------------------------------------------------------------- binding
    def _assign(self, items: Sequence[WorkItem], readers: int) -> tuple[tuple[int, ...], ...]:
        if self.assignment_policy is AssignmentPolicy.ROUND_ROBIN:
            return tuple(tuple(it.item_id for it in items if it.item_id % readers == r) for r in range(readers))
        total = sum(it.rows for it in items)
        out, cur, acc = [[] for _ in range(readers)], 0, 0
        for it in items:  # contiguous blocks, each close to total / readers rows
            if cur < readers - 1 and acc >= (cur + 1) * total / readers:
                cur += 1
            out[cur].append(it.item_id)
            acc += it.rows
        return tuple(tuple(x) for x in out)

    def build_scan_binding(self, world_size: int, *, cycle: Sequence[Sequence[int]] | None = None,
                           node_ids: Sequence[str] | None = None) -> SourceScanBinding:
        items = tuple(self.source_factory.plan())
        topo = self.build_reader_topology(world_size, cycle=cycle, node_ids=node_ids)
        return SourceScanBinding(items, plan_identity(items), 0, topo, self.tail_layout_mode(),
                                 self.assignment_policy, self._assign(items, world_size))

    # -------------------------------------------------------------- readers
    def create_session(self, *, pad_batch_factory=None):
        session = self.source_factory.create_session()
        if pad_batch_factory is not None:
            session.pad_batch_factory = pad_batch_factory
        return session

    def create_reader(self, rank: int, world_size: int, **kwargs: Any) -> BatchReader:
        """This rank's ``BatchReader`` (round-robin dealing of the planned items, per-reader batch)."""
        if self.assignment_policy is not AssignmentPolicy.ROUND_ROBIN:
            raise ValueError("BatchReader deals items round-robin; use the binding's assignments otherwise")
        topo = self.build_reader_topology(world_size)
        policy = CompletionPolicy.from_value(self.completion_policy).value
        return BatchReader(self.source_factory, topo.rows_per_reader(), rank=rank, world=world_size,
                           policy=policy, **kwargs)


__all__ = ["AssignmentPolicy", "RankDemand", "ReaderGroup", "ReaderTopology", "ScheduledDatasetSource",
           "SourceScanBinding", "TailLayoutMode", "plan_identity", "reader_worker_id", "tail_layout_mode"]
