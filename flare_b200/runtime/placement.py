"""Role resource profiles and rank placement over nodes.

On B200 the reference's Ray roles collapse into one process per GPU (input
stage, embedding-table owner and dense compute share it; reader lanes are
threads or CPU processes next to it), so placement decides:

* which node each GPU rank lives on: ranks fill nodes in contiguous blocks so
  that every tensor-parallel group (and, when it fits, every FSDP group) stays
  inside one NVLink domain;
* where the reader lanes run: lane ``l`` feeds input rank
  ``l // (readers / ranks)`` and is co-located with it (the reference's
  reader-lane = input-rank support constraint);
* how far each node's scalable roles grow (``ResourceScale`` steps, e.g.
  host memory for host-tier embedding tables): ``balanced`` raises the
  minimum weighted dominant share across nodes step by step, ``feasible``
  only checks capacity and maximises the minimum per-node occupancy.

Every role spans the same set of nodes (support equality), and capacity
(CPU, GPU, memory) is checked per node.  Reference behaviour:
src/flare/runtime/fluxway/placement/solver.py:39-119 and
src/flare/runtime/fluxway/resources/resolution.py:20-52,
recipes/recsys/ranking/resources.py:19-34 (default role profiles).
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Literal

GiB = 1024 ** 3
RESOURCES = ("CPU", "GPU", "memory")


@dataclass(frozen=True)
class ResourceScale:
    step: Mapping[str, float]
    max_steps: int = 0
    weight: float = 1.0


@dataclass(frozen=True)
class ResourceProfile:
    base: Mapping[str, float]
    scale: ResourceScale | None = None

    def demand(self, steps: int = 0) -> dict[str, float]:
        out = {k: float(self.base.get(k, 0)) for k in RESOURCES}
        if self.scale is not None and steps:
            if steps > self.scale.max_steps:
                raise ValueError(f"{steps} scale steps exceed max_steps {self.scale.max_steps}")
            for k, v in self.scale.step.items():
                out[k] = out.get(k, 0.0) + steps * float(v)
        return out


class ResourceProfiles:
    def __init__(self, roles: Mapping[str, ResourceProfile]):
        self._roles = dict(roles)

    def get_role(self, role: str) -> ResourceProfile:
        try:
            return self._roles[role]
        except KeyError as exc:
            raise KeyError(f"role {role!r} has no ResourceProfile") from exc

    def roles(self) -> list[str]:
        return list(self._roles)


# One GPU rank = input stage + table owner + dense compute; tables scale with host memory (host tier).
DEFAULT_ROLE_PROFILES: Mapping[str, ResourceProfile] = {
    "reader": ResourceProfile(base={"CPU": 1, "memory": 4 * GiB}),
    "rank": ResourceProfile(base={"CPU": 4, "GPU": 1, "memory": 16 * GiB},
                            scale=ResourceScale(step={"memory": 8 * GiB}, max_steps=255, weight=2.0)),
    "metrics": ResourceProfile(base={"CPU": 1, "memory": 2 * GiB}),
}
CPU_RANK_PROFILE = ResourceProfile(base={"CPU": 4, "memory": 16 * GiB},
                                   scale=ResourceScale(step={"memory": 8 * GiB}, max_steps=255, weight=2.0))


def resolve_resource_profiles(worker_counts: Mapping[str, int],
                              role_profiles: Mapping[str, ResourceProfile] = DEFAULT_ROLE_PROFILES, *,
                              compute_device: Literal["cpu", "gpu"] = "gpu",
                              device_overrides: Mapping[str, Mapping[str, ResourceProfile]] | None = None,
                              ) -> ResourceProfiles:
    """Validate a worker layout and pick each role's profile (device-specific override first)."""
    if compute_device not in ("cpu", "gpu"):
        raise ValueError(f"compute_device must be 'cpu' or 'gpu', got {compute_device!r}")
    bad = {r: c for r, c in worker_counts.items() if type(c) is not int or c <= 0}
    if bad:
        raise ValueError(f"worker counts must be positive integers: {bad}")
    missing = sorted(set(worker_counts) - set(role_profiles) - {"driver"})
    if missing:
        raise KeyError(f"worker roles have no ResourceProfile: {missing}")
    if device_overrides is None and compute_device == "cpu":
        device_overrides = {"cpu": {"rank": CPU_RANK_PROFILE}}
    over = (device_overrides or {}).get(compute_device, {})
    return ResourceProfiles({r: over.get(r, role_profiles[r]) for r in worker_counts if r in role_profiles})


@dataclass(frozen=True)
class NodeSpec:
    name: str
    cpus: float
    gpus: int
    memory: float

    def capacity(self) -> dict[str, float]:
        return {"CPU": float(self.cpus), "GPU": float(self.gpus), "memory": float(self.memory)}


@dataclass
class Placement:
    nodes: list[NodeSpec]
    rank_node: list[int]                 # node of every GPU rank
    reader_node: list[int]               # node of every reader lane
    reader_rank: list[int]               # input rank each reader lane feeds
    role_nodes: dict[str, list[int]]     # node of every worker of the other roles
    scale_steps: list[int]               # scale steps granted to each rank
    usage: list[dict[str, float]] = field(default_factory=list)

    def local_ranks(self) -> list[int]:
        """Local rank (GPU index) of every global rank on its node."""
        seen: dict[int, int] = {}
        out = []
        for n in self.rank_node:
            out.append(seen.get(n, 0))
            seen[n] = seen.get(n, 0) + 1
        return out

    def launch_plan(self) -> dict[str, list[tuple[int, int]]]:
        """Per node: (global rank, local rank) pairs, for one launcher per node."""
        plan: dict[str, list[tuple[int, int]]] = {n.name: [] for n in self.nodes}
        for r, (n, lr) in enumerate(zip(self.rank_node, self.local_ranks())):
            plan[self.nodes[n].name].append((r, lr))
        return plan


def _dominant_share(use: Mapping[str, float], cap: Mapping[str, float]) -> float:
    return max((use[k] / cap[k]) for k in RESOURCES if cap.get(k, 0) > 0)


def solve_placement(nodes: list[NodeSpec], worker_counts: Mapping[str, int], profiles: ResourceProfiles, *,
                    policy: Literal["balanced", "feasible"] = "balanced", tp: int = 1, fsdp: int = 1,
                    target_scale_steps: int | None = None) -> Placement:
    """Place ``rank`` workers (one per GPU), their reader lanes and the other roles on ``nodes``."""
    if policy not in ("balanced", "feasible"):
        raise ValueError(f"unknown placement policy: {policy!r}")
    ranks = worker_counts.get("rank", 0)
    readers = worker_counts.get("reader", ranks)
    if ranks <= 0:
        raise ValueError("at least one rank is required")
    if ranks % tp or ranks % (tp * fsdp) and fsdp > 1:
        raise ValueError(f"{ranks} ranks do not split into tensor-parallel groups of {tp} (x fsdp {fsdp})")
    if readers % ranks:
        raise ValueError("reader lanes must be a multiple of the ranks (each lane feeds one rank)")
    gpn = [n.gpus for n in nodes]
    if sum(gpn) < ranks and profiles.get_role("rank").demand()["GPU"] > 0:
        raise ValueError(f"{ranks} ranks need {ranks} GPUs; the nodes have {sum(gpn)}")
    # ---- ranks: contiguous blocks per node; tensor-parallel groups never straddle nodes
    rank_demand = profiles.get_role("rank").demand()
    rank_node: list[int] = []
    n_used = 0
    for i, n in enumerate(nodes):
        if len(rank_node) == ranks:
            break
        fit = n.gpus if rank_demand["GPU"] > 0 else ranks
        fit = min(fit, ranks - len(rank_node))
        if fit % tp and len(rank_node) + fit < ranks:
            fit -= fit % tp
        rank_node += [i] * fit
        n_used = i + 1
    if len(rank_node) < ranks:
        raise ValueError("not enough nodes for the ranks")
    for g in range(0, ranks, tp):
        if len(set(rank_node[g:g + tp])) != 1:
            raise ValueError(f"tensor-parallel group of ranks {g}..{g + tp - 1} straddles nodes")
    used = list(range(n_used))
    # ---- readers next to their rank, other roles round-robin over the used nodes (same support)
    factor = readers // ranks
    reader_rank = [lane // factor for lane in range(readers)]
    reader_node = [rank_node[r] for r in reader_rank]
    role_nodes: dict[str, list[int]] = {}
    for role, count in worker_counts.items():
        if role in ("rank", "reader", "driver"):
            continue
        role_nodes[role] = [used[k % len(used)] for k in range(count)]
    usage = [{k: 0.0 for k in RESOURCES} for _ in nodes]

    def add(node, dem, sign=1.0):
        for k in RESOURCES:
            usage[node][k] += sign * dem.get(k, 0.0)

    for r in range(ranks):
        add(rank_node[r], rank_demand)
    for lane in range(readers):
        add(reader_node[lane], profiles.get_role("reader").demand() if "reader" in profiles.roles() else {})
    for role, where in role_nodes.items():
        for n in where:
            add(n, profiles.get_role(role).demand())
    caps = [n.capacity() for n in nodes]
    for i in used:
        over = [k for k in RESOURCES if usage[i][k] > caps[i][k] + 1e-9]
        if over:
            raise ValueError(f"node {nodes[i].name}: base demand exceeds capacity in {over}")
    # support equality: every role touches every used node when it has enough workers
    for role, where in list(role_nodes.items()) + [("reader", reader_node)]:
        if len(where) >= len(used) and set(where) != set(used):
            raise ValueError(f"role {role} does not span the ranks' nodes")
    # ---- scale steps of the ranks
    scale = profiles.get_role("rank").scale
    steps = [0] * ranks
    if scale is not None and scale.max_steps > 0:
        step_dem = {k: float(scale.step.get(k, 0.0)) for k in RESOURCES}

        def fits(node):
            return all(usage[node][k] + step_dem[k] <= caps[node][k] + 1e-9 for k in RESOURCES)

        limit = scale.max_steps if target_scale_steps is None else min(scale.max_steps, target_scale_steps)
        while True:
            cands = [r for r in range(ranks) if steps[r] < limit and fits(rank_node[r])]
            if not cands:
                break
            if policy == "balanced":
                # the rank whose node has the lowest weighted dominant share grows first
                r = min(cands, key=lambda r: (scale.weight * _dominant_share(usage[rank_node[r]], caps[rank_node[r]]),
                                              steps[r], r))
            else:
                r = min(cands, key=lambda r: (steps[r], r))
            steps[r] += 1
            add(rank_node[r], step_dem)
        if policy == "feasible" and target_scale_steps is not None and min(steps) < target_scale_steps:
            raise ValueError(f"only {min(steps)} of {target_scale_steps} scale steps fit on every rank")
    return Placement(list(nodes), rank_node, reader_node, reader_rank, role_nodes, steps, usage)


__all__ = ["CPU_RANK_PROFILE", "DEFAULT_ROLE_PROFILES", "GiB", "NodeSpec", "Placement", "ResourceProfile",
           "ResourceProfiles", "ResourceScale", "resolve_resource_profiles", "solve_placement"]
