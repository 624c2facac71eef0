"""Framework-neutral training contracts.

These keep the reference's public names and fields on purpose so that code
written against the reference's contracts ports over unchanged:
ZeRO partition contracts (src/flare/training/zero/contracts.py:7-62), the
execution plan (src/flare/training/execution/plan.py:10-128), the optimizer
update window (src/flare/training/execution/update_window.py:12-74), the state
lifecycle (src/flare/training/state.py:8-51) and the task/batch/port schema
types (src/flare/training/contracts/*.py).
"""
from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from enum import Enum, IntEnum
from types import MappingProxyType
from typing import Any, Literal, Protocol


# ---------------------------------------------------------------- ZeRO
class ZeroStage(IntEnum):
    REPLICATED = 0
    OPTIMIZER_STATE = 1
    GRADIENT = 2
    PARAMETER = 3


@dataclass(frozen=True, slots=True)
class ZeroPartitionContract:
    """Which state is sharded and which collective moves gradients / parameters."""

    stage: ZeroStage
    axis_name: str
    parameter_partition: str
    optimizer_state_partition: str
    gradient_partition: str
    gradient_collective: str
    parameter_collective: str


_ZERO_TABLE = {
    # stage: (param, optimizer, grad, grad collective, param collective)
    ZeroStage.REPLICATED: ("replicated", "replicated", "replicated", "none", "none"),
    ZeroStage.OPTIMIZER_STATE: ("replicated", "sharded", "replicated", "all-reduce", "none"),
    ZeroStage.GRADIENT: ("replicated", "sharded", "sharded", "reduce-scatter", "all-gather"),
    ZeroStage.PARAMETER: ("sharded", "sharded", "sharded", "reduce-scatter", "all-gather"),
}


def zero_partition_contract(stage: ZeroStage, axis_name: str = "dp") -> ZeroPartitionContract:
    if not isinstance(stage, ZeroStage):
        raise TypeError(f"stage must be ZeroStage, got {type(stage).__name__}")
    if not axis_name:
        raise ValueError("axis_name must be non-empty")
    return ZeroPartitionContract(stage, axis_name, *_ZERO_TABLE[stage])


# ---------------------------------------------------------- execution plan
@dataclass(frozen=True, slots=True)
class ZeroExecutionPolicy:
    stage: ZeroStage
    axis_name: str = "dp"
    shard_scope: Literal["global", "node"] = "global"

    def __post_init__(self) -> None:
        if not isinstance(self.stage, ZeroStage):
            raise TypeError("stage must be a ZeroStage instance")
        if not self.axis_name:
            raise ValueError("axis_name must be non-empty")
        if self.shard_scope not in ("global", "node"):
            raise ValueError("shard_scope must be global or node")
        if self.shard_scope == "node" and self.stage is ZeroStage.REPLICATED:
            raise ValueError("node shard scope requires ZeRO stage 1, 2, or 3")


@dataclass(frozen=True, slots=True)
class GradientAccumulationPolicy:
    micro_steps: int = 1
    sync_mode: Literal["boundary", "micro"] = "boundary"

    def __post_init__(self) -> None:
        if self.micro_steps <= 0:
            raise ValueError("micro_steps must be positive")
        if self.sync_mode not in ("boundary", "micro"):
            raise ValueError("sync_mode must be boundary or micro")


@dataclass(frozen=True, slots=True)
class MacroUpdatePolicy:
    apply_optimizer_at_boundary: bool = True


@dataclass(frozen=True, slots=True)
class TrainingExecutionPlan:
    """Partitioning + accumulation + update policy of one training job."""

    zero: ZeroExecutionPolicy
    accumulation: GradientAccumulationPolicy
    update: MacroUpdatePolicy

    @classmethod
    def replicated(cls, *, micro_steps: int = 1, apply_optimizer_at_boundary: bool = True) -> "TrainingExecutionPlan":
        return cls(ZeroExecutionPolicy(ZeroStage.REPLICATED), GradientAccumulationPolicy(micro_steps),
                   MacroUpdatePolicy(apply_optimizer_at_boundary))

    @classmethod
    def sharded(cls, stage: ZeroStage, *, micro_steps: int = 1, sync_mode: str = "boundary",
             shard_scope: str = "global") -> "TrainingExecutionPlan":
        return cls(ZeroExecutionPolicy(stage, shard_scope=shard_scope), GradientAccumulationPolicy(micro_steps, sync_mode),
                   MacroUpdatePolicy(True))


@dataclass(frozen=True, slots=True)
class TrainingInputPlan:
    mode: Literal["manifest", "repeat_first_batch"]
    manifest_source_enabled: bool
    source_epochs: int
    checkpoint_enabled: bool
    checkpoint_reason: Literal["manifest_source", "existing_checkpoint", "scheduled", "disabled"]


def resolve_training_input_plan(*, reader_repeat_first_batch: bool, latest_checkpoint_step: int | None,
                                run_steps: int, target_step: int, checkpoint_interval_steps: int) -> TrainingInputPlan:
    """Decide the input mode and whether checkpointing is on.

    Repeat-first-batch is a simulation mode: it cannot restore a checkpoint and
    replays one batch for ``target_step`` epochs.
    """
    if not isinstance(reader_repeat_first_batch, bool):
        raise TypeError("reader_repeat_first_batch must be a boolean")
    for name, v in (("run_steps", run_steps), ("target_step", target_step),
                    ("checkpoint_interval_steps", checkpoint_interval_steps)):
        if v <= 0:
            raise ValueError(f"{name} must be positive, got {v}")
    if latest_checkpoint_step is not None and (isinstance(latest_checkpoint_step, bool) or latest_checkpoint_step < 0):
        raise ValueError(f"latest_checkpoint_step must be non-negative when provided, got {latest_checkpoint_step}")
    if reader_repeat_first_batch and latest_checkpoint_step is not None:
        raise ValueError("reader_repeat_first_batch simulation mode cannot restore a checkpoint")
    manifest = not reader_repeat_first_batch
    if latest_checkpoint_step is not None:
        enabled, reason = True, "existing_checkpoint"
    elif checkpoint_interval_steps <= run_steps:
        enabled, reason = True, "scheduled"
    else:
        enabled, reason = False, "disabled"
    return TrainingInputPlan("manifest" if manifest else "repeat_first_batch", manifest,
                             1 if manifest else target_step, enabled, reason)


# --------------------------------------------------------- update window
@dataclass(frozen=True, slots=True)
class OptimizerUpdateWindow:
    """Identity of one optimizer window, shared by dense and sparse updates."""

    micro_step: int
    accumulation_steps: int
    at_boundary: bool
    should_apply_update: bool
    optimizer_step: int

    def __post_init__(self) -> None:
        if self.micro_step <= 0:
            raise ValueError("micro_step must be positive")
        if self.accumulation_steps <= 0:
            raise ValueError("accumulation_steps must be positive")
        if self.micro_step > self.accumulation_steps:
            raise ValueError("micro_step cannot exceed accumulation_steps")
        if self.optimizer_step < 0:
            raise ValueError("optimizer_step must be non-negative")
        if self.at_boundary != (self.micro_step == self.accumulation_steps):
            raise ValueError("at_boundary must equal the accumulation boundary state")
        if self.should_apply_update and not self.at_boundary:
            raise ValueError("an update can only apply at an accumulation boundary")

    def encode(self) -> tuple[int, int, int, int, int]:
        """Five integers, the stable wire form used between roles."""
        return (self.micro_step, self.accumulation_steps, int(self.at_boundary), int(self.should_apply_update),
                self.optimizer_step)

    @classmethod
    def decode(cls, values: Sequence[int]) -> "OptimizerUpdateWindow":
        if len(values) != 5:
            raise ValueError("encoded OptimizerUpdateWindow must contain exactly five integers")
        m, a, b, s, o = (int(v) for v in values)
        if b not in (0, 1) or s not in (0, 1):
            raise ValueError("encoded OptimizerUpdateWindow boolean fields must be 0 or 1")
        return cls(m, a, bool(b), bool(s), o)


# ------------------------------------------------------------- lifecycle
@dataclass(frozen=True, slots=True)
class TrainingStateBlueprint:
    groups: tuple[str, ...]
    leaves: tuple[tuple[str, tuple[int, ...], str, str], ...]
    schema_digest: str

    def __post_init__(self) -> None:
        if not self.groups or len(self.groups) != len(set(self.groups)):
            raise ValueError("TrainingStateBlueprint groups must be unique and non-empty")
        if not self.leaves:
            raise ValueError("TrainingStateBlueprint requires at least one leaf")
        if not self.schema_digest:
            raise ValueError("TrainingStateBlueprint schema_digest must be non-empty")
        paths = [leaf[0] for leaf in self.leaves]
        if len(paths) != len(set(paths)):
            raise ValueError("TrainingStateBlueprint leaf paths must be unique")
        for path, shape, dtype, role in self.leaves:
            if not path or any(int(d) < 0 for d in shape):
                raise ValueError("TrainingStateBlueprint leaf shape is invalid")
            if not dtype or not role:
                raise ValueError("TrainingStateBlueprint leaf dtype and role are required")


class TrainingStateLifecycle(str, Enum):
    """Where a training state's concrete values come from."""

    FRESH_INITIALIZE = "fresh_initialize"
    CHECKPOINT_RESTORE = "checkpoint_restore"
    MODEL_WEIGHTS = "model_weights"


# ------------------------------------------------------- task / schema
@dataclass(frozen=True)
class TensorSpec:
    shape: tuple[int | None, ...]
    dtype: str

    def __post_init__(self) -> None:
        if not self.dtype:
            raise ValueError("TensorSpec dtype cannot be empty")


@dataclass(frozen=True)
class PortSpec:
    name: str
    spec: TensorSpec | None = None
    is_optional: bool = False

    def __post_init__(self) -> None:
        if not self.name:
            raise ValueError("PortSpec name cannot be empty")


@dataclass(frozen=True)
class BatchFieldSpec:
    name: str
    spec: TensorSpec
    is_sparse: bool = False
    is_label: bool = False
    is_weight: bool = False


@dataclass(frozen=True)
class BatchSchema:
    fields: Mapping[str, BatchFieldSpec]

    def __getitem__(self, name: str) -> BatchFieldSpec:
        return self.fields[name]

    def __contains__(self, name: str) -> bool:
        return name in self.fields


@dataclass(frozen=True)
class PayloadField:
    name: str
    dtype: str
    shape: tuple[int | None, ...]
    optional: bool = False
    is_dynamic: bool = False

    def __post_init__(self) -> None:
        if not self.name or not isinstance(self.name, str):
            raise ValueError(f"PayloadField requires non-empty name, got {self.name!r}")
        if not self.dtype or not isinstance(self.dtype, str):
            raise ValueError(f"PayloadField requires non-empty dtype, got {self.dtype!r}")
        if not isinstance(self.shape, tuple):
            raise TypeError("PayloadField shape must be a tuple")


@dataclass(frozen=True)
class PayloadSchema:
    name: str
    fields: tuple[PayloadField, ...]

    def __post_init__(self) -> None:
        if not self.name:
            raise ValueError("PayloadSchema requires a non-empty name")
        if not isinstance(self.fields, tuple):
            raise TypeError("PayloadSchema fields must be a tuple")
        seen = set()
        for f in self.fields:
            if not isinstance(f, PayloadField):
                raise TypeError(f"Field must be PayloadField, got {type(f).__name__}")
            if f.name in seen:
                raise ValueError(f"Duplicate field name {f.name!r} in PayloadSchema {self.name!r}")
            seen.add(f.name)

    @property
    def field_names(self) -> tuple[str, ...]:
        return tuple(f.name for f in self.fields)


@dataclass(frozen=True)
class TaskSpec:
    name: str
    batch_schema: BatchSchema
    output_ports: tuple[PortSpec, ...]
    loss: Callable[[Any, Any], Any]
    metrics: Mapping[str, Any] | None = None
    properties: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not self.name or not isinstance(self.name, str):
            raise ValueError(f"TaskSpec requires non-empty name, got {self.name!r}")
        if not isinstance(self.batch_schema, BatchSchema):
            raise TypeError("TaskSpec batch_schema must be BatchSchema")
        if not callable(self.loss):
            raise TypeError("TaskSpec loss must be callable")


class BatchEvaluator(Protocol):
    def evaluate_batch(self, batch: Any) -> Any: ...


@dataclass(frozen=True)
class EvaluationEnvelope:
    payload: Any
    request_id: str
    schema_id: str
    metadata: Mapping[str, Any]

    def __post_init__(self) -> None:
        if not isinstance(self.request_id, str) or not self.request_id:
            raise ValueError("EvaluationEnvelope request_id must be a non-empty string")
        if not isinstance(self.schema_id, str) or not self.schema_id:
            raise ValueError("EvaluationEnvelope schema_id must be a non-empty string")
        if not isinstance(self.metadata, MappingProxyType):
            raise TypeError("EvaluationEnvelope metadata must be a MappingProxyType")

    @classmethod
    def from_metadata(cls, *, payload: Any, request_id: str, schema_id: str,
                      metadata: Mapping[str, Any]) -> "EvaluationEnvelope":
        return cls(payload, request_id, schema_id, MappingProxyType(dict(metadata)))


__all__ = [
    "BatchEvaluator", "BatchFieldSpec", "BatchSchema", "EvaluationEnvelope", "GradientAccumulationPolicy",
    "MacroUpdatePolicy", "OptimizerUpdateWindow", "PayloadField", "PayloadSchema", "PortSpec", "TaskSpec",
    "TensorSpec", "TrainingExecutionPlan", "TrainingInputPlan", "TrainingStateBlueprint", "TrainingStateLifecycle",
    "ZeroExecutionPolicy", "ZeroPartitionContract", "ZeroStage", "resolve_training_input_plan",
    "zero_partition_contract",
]
