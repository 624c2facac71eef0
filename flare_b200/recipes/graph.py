"""Ranking graph assembly and phase schedule for the fused B200 path.

The reference assembles a Fluxway task graph of Ray roles (reader -> input
-> sparse tables -> train -> metrics) and schedules each training step as a
set of phases on a compute and a data lane
(recipes/recsys/ranking/topology.py:311-417, graph/pipeline.py:74-255,
workers/schedule.py:7-40).  Here every role is part of one process per GPU,
so the same assembly produces nodes in-process:

* reader: a host prefetch loader (pinned batches, async host -> device copy);
* input: the step's static buffers (dense features, labels) and the fused
  collection's exchange buffers (keyed-jagged ids);
* tables: the fused sharded embedding collection (``FusedEmbeddingBag``);
* train: the user module on the flat fused optimizer, one CUDA graph per step;
* metrics: device metric windows (exact AUC / calibration / loss per target).

``RankingTaskGraph.run(steps)`` executes each step as the schedule's phases in
dependency order and records their host time.  The phase contract (names,
lanes, priorities, dependencies with their step distance) is a table the
step follows; in the fused step the sparse-gradient scatter and the dense
update run inside ``train_core``'s graph (the lookup's backward and the fused
optimizer), so their phases only mark where they happened.
"""
from __future__ import annotations

import time
from collections.abc import Iterable, Mapping
from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass(frozen=True)
class PhaseSpec:
    name: str
    lane: str
    priority: int


# the step's phases, in order (lane: which queue the reference runs them on; priority: its tie-break)
RANKING_PHASES = (
    PhaseSpec("prepare_sparse_materialize", "data", 300),
    PhaseSpec("prepare_bind", "data", 290),
    PhaseSpec("train_core", "compute", 500),
    PhaseSpec("scatter_sparse_grads", "data", 20),
    PhaseSpec("update", "compute", 480),
    PhaseSpec("materialize_train_metrics", "data", 10),
)
RANKING_PHASE_ORDER = tuple(p.name for p in RANKING_PHASES)
RANKING_LANE_ORDER = ("compute", "data")
RANKING_LANE_PRIORITIES = {"compute": 1000, "data": 100}
RANKING_PHASE_LANES = {p.name: p.lane for p in RANKING_PHASES}
RANKING_PHASE_PRIORITIES = {p.name: p.priority for p in RANKING_PHASES}
# (before, after, step distance): "update" of step t precedes "train_core" of step t+1
RANKING_PHASE_DEPENDENCIES = (
    ("prepare_sparse_materialize", "prepare_bind", 0),
    ("prepare_bind", "train_core", 0),
    ("train_core", "scatter_sparse_grads", 0),
    ("train_core", "update", 0),
    ("train_core", "materialize_train_metrics", 0),
    ("update", "train_core", 1),
)


def schedule_order(phases=RANKING_PHASES, deps=RANKING_PHASE_DEPENDENCIES) -> tuple[str, ...]:
    """Phases of one step in an order that meets every same-step dependency (ties: higher priority
    first, then compute before data)."""
    names = [p.name for p in phases]
    spec = {p.name: p for p in phases}
    preds = {n: {a for a, b, d in deps if b == n and d == 0} for n in names}
    out: list[str] = []
    while len(out) < len(names):
        ready = [n for n in names if n not in out and preds[n] <= set(out)]
        if not ready:
            raise ValueError("the phase dependencies have a cycle within one step")
        ready.sort(key=lambda n: (-spec[n].priority, RANKING_LANE_ORDER.index(spec[n].lane)))
        out.append(ready[0])
    return tuple(out)


@dataclass
class PipelineInputs:
    """The assembled non-training nodes (the reference's ``PipelineInputs``)."""
    tables: Any            # FusedEmbeddingBag
    model_arguments: Mapping[str, Any]
    processed: Any         # the step's static device buffers
    reader: Any            # batch source (host)
    input_node: Any        # moves a batch into the static buffers
    trainer: Any = None


@dataclass
class _InputNode:
    trainer: Any

    def step(self, batch) -> None:
        dense, labels, offsets, values = batch
        self.trainer.set_batch(dense, labels, offsets, values)


def build_pipeline_nodes(recipe, *, source: Iterable, rank: int = 0, world_size: int = 1,
                         device: torch.device | None = None, use_graph: bool = True, seed: int = 0,
                         trainer_kwargs: Mapping[str, Any] | None = None) -> PipelineInputs:
    """Reader, input and table nodes for ``recipe`` (and the trainer that owns the step buffers).

    ``source`` yields ``(dense, label_ids, offsets, values)`` of this rank's local batch."""
    trainer = recipe.trainer(rank=rank, world_size=world_size, device=device, use_graph=use_graph, seed=seed,
                             **dict(trainer_kwargs or {}))
    return PipelineInputs(
        tables=trainer.emb,
        model_arguments={"dense": trainer.x_dense, "pooled": "tables.forward()"},
        processed={"dense": trainer.x_dense, "label_ids": trainer.label_ids},
        reader=iter(source),
        input_node=_InputNode(trainer),
        trainer=trainer,
    )


@dataclass
class RankingTaskGraph:
    inputs: PipelineInputs
    metrics: Any = None
    order: tuple[str, ...] = field(default_factory=schedule_order)
    phase_seconds: dict[str, float] = field(default_factory=dict)
    steps_run: int = 0
    losses: list[float] = field(default_factory=list)

    def run(self, steps: int, *, read_loss_every: int = 1, trace=None) -> list[float]:
        """Run ``steps`` training steps; returns the losses read back (every ``read_loss_every`` steps;
        0: never, so the host runs ahead of the GPU).  ``trace`` (a ``validation.perfetto.PerfettoWriter``)
        receives one slice per phase and step on ``rank:<r>/<lane>`` tracks: host phases as measured on
        the host, ``train_core`` as its device interval (CUDA events around the step's graph)."""
        tr = self.inputs.trainer
        lane = {p.name: p.lane for p in RANKING_PHASES}
        rank_track = f"rank:{tr.rank}"
        dev_marks = []
        if trace is not None:
            torch.cuda.synchronize(tr.device)
            host0 = time.perf_counter_ns()
            base = torch.cuda.Event(enable_timing=True)
            base.record()
        for _ in range(steps):
            step = self.steps_run
            batch = None
            loss = None
            for phase in self.order:
                t0 = time.perf_counter_ns()
                if phase == "prepare_sparse_materialize":
                    batch = next(self.inputs.reader)
                elif phase == "prepare_bind":
                    self.inputs.input_node.step(batch)
                elif phase == "train_core":
                    if trace is not None:
                        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        ea.record()
                    loss = tr._run()  # forward, backward (fused sparse update inside), fused dense update
                    tr.steps += 1
                    if trace is not None:
                        eb.record()
                        dev_marks.append((step, ea, eb))
                elif phase == "materialize_train_metrics" and self.metrics is not None:
                    logits = self.metrics.logits_fn()
                    self.metrics.window.update(logits, self.metrics.labels_fn(), loss_sum=loss * tr.global_B)
                # scatter_sparse_grads and update ran inside train_core's graph
                t1 = time.perf_counter_ns()
                self.phase_seconds[phase] = self.phase_seconds.get(phase, 0.0) + (t1 - t0) / 1e9
                if trace is not None and phase != "train_core":
                    trace.slice((rank_track, lane[phase]), phase, t0, t1, step=step, lane=lane[phase])
            self.steps_run += 1
            if read_loss_every and self.steps_run % read_loss_every == 0:
                self.losses.append(float(loss.item()))
        if trace is not None:
            torch.cuda.synchronize(tr.device)
            for step, ea, eb in dev_marks:
                a = host0 + int(base.elapsed_time(ea) * 1e6)
                b = host0 + int(base.elapsed_time(eb) * 1e6)
                trace.slice((rank_track, "compute"), "train_core", a, b, step=step, lane="compute")
        return self.losses


@dataclass
class _MetricsNode:
    window: Any
    logits_fn: Any
    labels_fn: Any


def assemble_ranking_training_graph(graph_inputs: PipelineInputs, *,
                                    metrics_static_args: Mapping[str, Any] | None = None) -> dict[str, Any]:
    """Training graph of the assembled nodes: ``{"training", "metrics", "placement", "task_graph"}``.

    With ``metrics_static_args`` (``TrainMetricsWindow`` arguments) each step's per-target predictions
    go into a device metric window; its logits come from one extra forward of the step's batch."""
    tr = graph_inputs.trainer
    metrics = None
    if metrics_static_args is not None:
        from ..metrics.aggregation import TrainMetricsWindow

        objective = tr.objective
        window = TrainMetricsWindow(device=tr.device, **dict(metrics_static_args))

        def logits_fn():
            with torch.no_grad():
                pooled = tr.emb.coll.pooled_output
                return tr.module(tr.x_dense, pooled, tr.emb.split(pooled))

        def labels_fn():
            return objective.per_target(tr.label_ids)[0]

        metrics = _MetricsNode(window, logits_fn, labels_fn)
    task_graph = RankingTaskGraph(graph_inputs, metrics)
    placement = {"rank": tr.rank, "world_size": tr.world, "roles": ("reader", "input", "tables", "train", "metrics"),
                 "device": str(tr.device)}
    return {"training": tr, "metrics": metrics, "placement": placement, "task_graph": task_graph}


@dataclass
class RankingEvalGraph:
    inputs: PipelineInputs

    def run(self, steps: int) -> dict[str, float]:
        """Predict ``steps`` batches; exact AUC per target and the mean prediction (calibration input)."""
        from ..metrics.ranking import auc

        tr = self.inputs.trainer
        scores, labels = [], []
        for _ in range(steps):
            dense, lab, offs, vals = next(self.inputs.reader)
            scores.append(tr.predict(dense, offs, vals))
            labels.append(tr.objective.per_target(lab.to(tr.device))[0])
        s, y = torch.cat(scores), torch.cat(labels)
        out = {}
        for t, name in enumerate(getattr(tr.objective, "targets", range(s.shape[1]))):
            out[f"auc/{name}"] = auc(s[:, t].contiguous(), y[:, t].contiguous())
            out[f"mean_prediction/{name}"] = float(s[:, t].mean())
            out[f"mean_label/{name}"] = float(y[:, t].mean())
        return out


def assemble_ranking_evaluation_graph(graph_inputs: PipelineInputs) -> dict[str, Any]:
    """Evaluation graph: ``{"evaluation", "task_graph"}`` (``task_graph.run(steps)`` -> metrics)."""
    return {"evaluation": graph_inputs.trainer, "task_graph": RankingEvalGraph(graph_inputs)}


__all__ = ["PhaseSpec", "PipelineInputs", "RANKING_LANE_ORDER", "RANKING_LANE_PRIORITIES", "RANKING_PHASES",
           "RANKING_PHASE_DEPENDENCIES", "RANKING_PHASE_LANES", "RANKING_PHASE_ORDER", "RANKING_PHASE_PRIORITIES",
           "RankingEvalGraph", "RankingTaskGraph", "assemble_ranking_evaluation_graph",
           "assemble_ranking_training_graph", "build_pipeline_nodes", "schedule_order"]
