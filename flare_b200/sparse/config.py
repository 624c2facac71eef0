"""Sparse table and optimizer configuration.

``SparseOptimizerConfig`` and ``SparseTableSpec`` keep the reference's field
names (src/flare/training/components/sparse_table/contracts.py:15-46).  The
optimizer kinds and dynamic learning-rate policies are implemented inside the
fused backward kernel (embedding.cu ``apply_row_update`` / ``lr_scale``); the
reference delegates them to its external native store, so their formulas are
defined here:

* ``constant``: lr
* ``sqrt_decay``: lr / sqrt(max(score, 1))
* ``log_decay``: lr / (1 + ln(1 + score))
* ``inverse_decay``: lr / max(score, 1)
* ``cosine_frequency``: lr * (r + (1 - r) * (1 + cos(pi * min(score, S) / S)) / 2)
  with r = ``cosine_min_lr_ratio`` and S = ``cosine_max_score``
* ``custom_lut``: lr * lut[min(floor(score), len(lut) - 1)]

where ``score`` is the row's cumulative occurrence count (its LFU score),
updated before the learning rate is computed.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

from .precision import (
    require_sparse_gradient_dtype,
    require_sparse_gradient_transport_dtype,
    require_sparse_optimizer_dtype,
    require_sparse_value_dtype,
)

OPTIMIZER_KINDS = {"sgd": 0, "rowwise_adagrad": 1, "adam": 2, "rowwise_adam": 3, "adagrad": 4}
LR_POLICIES = {"constant": 0, "sqrt_decay": 1, "log_decay": 2, "inverse_decay": 3, "cosine_frequency": 4,
               "custom_lut": 5}


@dataclass(frozen=True)
class SparseOptimizerConfig:
    kind: str = "rowwise_adagrad"
    learning_rate: float = 0.01
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.0
    dynamic_lr_policy: str = "constant"
    cosine_min_lr_ratio: float = 0.0
    cosine_max_score: float = 1.0
    custom_lut: tuple[float, ...] = ()

    def __post_init__(self) -> None:
        if self.kind not in OPTIMIZER_KINDS:
            raise ValueError(f"unsupported sparse optimizer {self.kind!r}")
        if self.dynamic_lr_policy not in LR_POLICIES:
            raise ValueError(f"unsupported sparse dynamic learning-rate policy {self.dynamic_lr_policy!r}")
        if self.dynamic_lr_policy == "custom_lut" and not self.custom_lut:
            raise ValueError("custom_lut policy needs a non-empty lut")
        if self.learning_rate < 0:
            raise ValueError("learning_rate must be non-negative")

    @property
    def needs_row_state(self) -> bool:
        return self.kind in ("rowwise_adagrad", "rowwise_adam")

    @property
    def needs_m(self) -> bool:
        return self.kind in ("adam", "rowwise_adam", "adagrad")

    @property
    def needs_v(self) -> bool:
        return self.kind == "adam"

    @property
    def needs_score(self) -> bool:
        return self.dynamic_lr_policy != "constant"

    def kernel_params(self, step: int) -> dict:
        """Scalar parameter block for the fused kernel at optimizer step ``step`` (1-based)."""
        t = max(int(step), 1)
        return dict(
            kind=OPTIMIZER_KINDS[self.kind], lr=float(self.learning_rate), beta1=float(self.beta1),
            beta2=float(self.beta2), eps=float(self.eps), weight_decay=float(self.weight_decay),
            bias_corr1=1.0 - math.pow(self.beta1, t), bias_corr2=1.0 - math.pow(self.beta2, t),
            lr_policy=LR_POLICIES[self.dynamic_lr_policy], policy_a=float(self.cosine_min_lr_ratio),
            policy_b=float(self.cosine_max_score),
        )


@dataclass(frozen=True)
class SparseTableSpec:
    """One logical embedding table.

    ``num_embeddings`` rows of width ``embedding_dim`` fed by input feature
    ``feature`` (defaults to the table name).  ``pooling`` is ``sum`` or
    ``mean``.  Dtype fields keep the reference's names and contracts.
    """

    name: str
    num_embeddings: int
    embedding_dim: int
    feature: str | None = None
    pooling: str = "sum"
    value_dtype: str = "float32"
    gradient_transport_dtype: str = "bfloat16"
    gradient_dtype: str = "float32"
    optimizer_dtype: str = "float32"
    optimizer: SparseOptimizerConfig = field(default_factory=SparseOptimizerConfig)
    init_scale: float = 0.01
    shards: int = 1                # > 1: row-wise pieces by key modulo (piece r holds rows i % shards == r)
    max_staleness_steps: int = 0   # lookups may miss this many recent updates (>= 1 everywhere: pipelined step)
    cache_rows: int | None = None  # host-DRAM tier: rows live in pinned host memory, this many in an HBM cache
    dynamic: bool = False          # hash-keyed: any int32 key >= 0, num_embeddings slots, insert on first sight
    hash_buckets: int | None = None  # dynamic: power-of-two hash buckets (default 4 x slots rounded up)

    def __post_init__(self) -> None:
        require_sparse_value_dtype(self.value_dtype)
        require_sparse_gradient_transport_dtype(self.gradient_transport_dtype)
        require_sparse_gradient_dtype(self.gradient_dtype)
        require_sparse_optimizer_dtype(self.optimizer_dtype)
        if self.num_embeddings <= 0 or self.embedding_dim <= 0:
            raise ValueError("table shape must be positive")
        if self.embedding_dim % 4:
            raise ValueError("embedding_dim must be a multiple of 4")
        if self.shards < 1:
            raise ValueError("shards must be >= 1")
        if self.shards > 1 and (self.dynamic or self.cache_rows is not None):
            raise ValueError("row-wise pieces (shards > 1) are for resident static tables")
        if self.dynamic and self.cache_rows is not None:
            raise ValueError("a table is either dynamic or host-tier, not both")
        if self.cache_rows is not None:
            if not 0 < self.cache_rows <= self.num_embeddings:
                raise ValueError("cache_rows must be in (0, num_embeddings]")
            if self.value_dtype != "float32":
                raise ValueError("host-tier tables store fp32 rows")
        if self.pooling not in ("sum", "mean"):
            raise ValueError(f"unsupported pooling {self.pooling!r}")
        if isinstance(self.max_staleness_steps, bool) or self.max_staleness_steps < 0:
            raise ValueError(f"max_staleness_steps must be non-negative, got {self.max_staleness_steps}")

    @property
    def feature_name(self) -> str:
        return self.feature or self.name


__all__ = ["LR_POLICIES", "OPTIMIZER_KINDS", "SparseOptimizerConfig", "SparseTableSpec"]
