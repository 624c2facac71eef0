"""Batch schema: ragged feature batches, feature layout, Arrow -> training dict.

Behaviour follows the reference's schema layer (src/flare/data/schema/
batch.py:9, feature_layout.py:16-142, transform.py:333, virtual_pad.py:12):

* ``RaggedFeatureBatch`` = flat values + int32 nested row splits, validated
  (monotonic, starting at 0, ending at the number of values);
* ``TrainingFeatureLayout`` maps logical feature names to physical columns and
  defines the null sentinel;
* ``table_to_training_dict`` turns an Arrow table into the training payload:
  a side-info int32 matrix (categorical ids shifted by +1 so null -> 0), one
  keyed-jagged sparse group per configured group (feature-major offsets and
  values, the layout the fused embedding kernels read), labels and metadata;
* ``virtual_pad`` pads a batch to a fixed row count and reports the valid
  prefix length.
"""
from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field

import numpy as np

try:  # pyarrow is optional at import time (only needed for Arrow inputs)
    import pyarrow as pa
except ImportError:  # pragma: no cover
    pa = None


@dataclass(frozen=True)
class RaggedFeatureBatch:
    flat_values: np.ndarray
    nested_splits: tuple[np.ndarray, ...]

    def __post_init__(self) -> None:
        if not self.nested_splits:
            raise ValueError("RaggedFeatureBatch needs at least one split level")
        inner = len(self.flat_values)
        for level in reversed(self.nested_splits):
            s = np.asarray(level)
            if s.dtype != np.int32:
                raise TypeError("row splits must be int32")
            if s.ndim != 1 or len(s) == 0 or s[0] != 0:
                raise ValueError("row splits must be 1-D and start at 0")
            if np.any(np.diff(s) < 0):
                raise ValueError("row splits must be non-decreasing")
            if int(s[-1]) != inner:
                raise ValueError(f"row splits end at {int(s[-1])}, expected {inner}")
            inner = len(s) - 1

    @property
    def nrows(self) -> int:
        return len(self.nested_splits[0]) - 1

    def row_lengths(self, level: int = -1) -> np.ndarray:
        return np.diff(self.nested_splits[level])


@dataclass(frozen=True)
class TrainingFeatureLayout:
    """Logical feature -> physical Arrow column (and null sentinel)."""

    columns: Mapping[str, str]
    null_value: int = -1
    categorical: tuple[str, ...] = ()
    dense: tuple[str, ...] = ()

    def column(self, feature: str) -> str:
        try:
            return self.columns[feature]
        except KeyError as exc:
            raise KeyError(f"feature {feature!r} is not in the training layout") from exc


@dataclass
class TrainingDict:
    side_info: np.ndarray | None
    dense: np.ndarray | None
    sparse: dict[str, tuple[np.ndarray, np.ndarray]]  # group -> (offsets int32 [F*B+1], values)
    labels: np.ndarray | None
    metadata: dict[str, np.ndarray] = field(default_factory=dict)

    @property
    def batch_size(self) -> int:
        for a in (self.side_info, self.dense, self.labels):
            if a is not None:
                return a.shape[0]
        for off, _ in self.sparse.values():
            return 0 if off is None else (len(off) - 1)
        return 0


def keyed_jagged_from_lists(per_feature: Sequence[Sequence[Sequence[int]]], dtype=np.int32):
    """[[ids of sample 0, ids of sample 1, ...] per feature] -> (offsets [F*B+1], values)."""
    lengths, vals = [], []
    for feat in per_feature:
        for ids in feat:
            lengths.append(len(ids))
            vals.extend(ids)
    offsets = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=offsets[1:])
    return offsets, np.asarray(vals, dtype=dtype)


def _list_column(col) -> tuple[np.ndarray, np.ndarray]:
    """Arrow list (or scalar) column -> (row lengths, flat values); nulls are empty lists."""
    if pa is not None and isinstance(col, pa.ChunkedArray):
        col = col.combine_chunks()
    if pa is not None and pa.types.is_list(col.type):
        offsets = np.asarray(col.offsets, dtype=np.int64)
        lengths = np.diff(offsets)
        valid = np.asarray(col.is_valid())
        lengths = np.where(valid, lengths, 0)
        flat = np.asarray(col.values.fill_null(-1))
        if not valid.all():
            keep = np.repeat(valid, np.diff(offsets))
            flat = flat[keep]
        else:
            flat = flat[offsets[0]:offsets[-1]]
        return lengths.astype(np.int64), flat
    arr = np.asarray(col.fill_null(-1) if pa is not None else col)
    lengths = (arr >= 0).astype(np.int64)
    return lengths, arr[arr >= 0]


def table_to_training_dict(table, layout: TrainingFeatureLayout, *,
                           sparse_groups: Mapping[str, Sequence[str]] | None = None,
                           label_column: str | None = None, metadata_columns: Sequence[str] = ()) -> TrainingDict:
    """Arrow table -> training payload (see module docstring)."""
    B = table.num_rows
    side = None
    if layout.categorical:
        side = np.zeros((B, len(layout.categorical)), dtype=np.int32)
        for j, feat in enumerate(layout.categorical):
            col = table.column(layout.column(feat))
            vals = np.asarray(col.fill_null(layout.null_value)).astype(np.int64)
            side[:, j] = np.where(vals == layout.null_value, 0, vals + 1).astype(np.int32)
    dense = None
    if layout.dense:
        dense = np.stack([np.asarray(table.column(layout.column(f)).fill_null(0.0), dtype=np.float32)
                          for f in layout.dense], 1)
    sparse = {}
    for group, feats in (sparse_groups or {}).items():
        lens, vals = [], []
        for f in feats:
            ln, fl = _list_column(table.column(layout.column(f)))
            lens.append(ln)
            vals.append(fl)
        lengths = np.concatenate(lens) if lens else np.zeros(0, np.int64)
        offsets = np.zeros(len(lengths) + 1, dtype=np.int64)
        np.cumsum(lengths, out=offsets[1:])
        sparse[group] = (offsets.astype(np.int32), np.concatenate(vals).astype(np.int32) if vals else
                         np.zeros(0, np.int32))
    labels = None
    if label_column is not None:
        labels = np.asarray(table.column(label_column).fill_null(0), dtype=np.float32).reshape(B, -1)
    meta = {c: np.asarray(table.column(c)) for c in metadata_columns}
    return TrainingDict(side, dense, sparse, labels, meta)


def virtual_pad(td: TrainingDict, rows: int) -> tuple[TrainingDict, int]:
    """Pad a training dict to ``rows`` samples; returns (padded, valid_count)."""
    B = td.batch_size
    if rows < B:
        raise ValueError(f"cannot pad {B} rows down to {rows}")
    pad = rows - B

    def pad_rows(a, fill=0):
        if a is None:
            return None
        return np.concatenate([a, np.full((pad,) + a.shape[1:], fill, dtype=a.dtype)])

    sparse = {}
    for g, (off, vals) in td.sparse.items():
        F = (len(off) - 1) // max(B, 1) if B else 0
        lens = np.diff(off).reshape(F, B) if B else np.zeros((F, 0), np.int32)
        lens = np.concatenate([lens, np.zeros((F, pad), dtype=lens.dtype)], 1).reshape(-1)
        new_off = np.zeros(len(lens) + 1, dtype=np.int32)
        np.cumsum(lens, out=new_off[1:])
        sparse[g] = (new_off, vals)
    return TrainingDict(pad_rows(td.side_info), pad_rows(td.dense), sparse, pad_rows(td.labels),
                        {k: pad_rows(v) for k, v in td.metadata.items()}), B


__all__ = ["RaggedFeatureBatch", "TrainingDict", "TrainingFeatureLayout", "keyed_jagged_from_lists",
           "table_to_training_dict", "virtual_pad"]
