"""Ranking recipe schema helpers: batch contract, sparse-group naming, padded inverse indices.

* ``RankingBatch`` / ``build_ranking_batch_schema``: the fields a ranking
  step consumes (one int64 ragged field per sparse group, float side-info
  matrices, int32 labels, optional group ids, the valid-sample count) on
  the framework's ``BatchSchema`` contract.
* Sparse groups are named ``<base>_dim_<d>`` (the embedding width in the
  name): ``parse_sparse_group_name``, ``extract_sparse_groups_and_dimensions``
  (base -> sorted widths), ``extract_sparse_base_names``; per-group counts
  from a knob string (``"4"`` for every base, or ``"users:2,items:1"``) with
  ``parse_sparse_workers`` (default 1) and ``parse_sparse_thread_budgets``
  (only the named ones); ``build_sparse_group_feature_widths`` gives each
  group's (features, widest feature) from the model's feature groups.
* ``materialize_padded_inverse``: a ragged inverse index (a dense prefix
  matrix, or flat values with nested row splits) into a dense
  ``[batch, *target_widths]`` array filled with ``pad_index``; elements past
  a target width are dropped; ``audit=True`` checks the splits (start at 0,
  monotone, ending at the child count), the shapes and the index range
  before writing.  Vectorised: each nesting level maps the flat positions of
  its children to ``parent * width + local`` in one pass.

The fused kernels read keyed-jagged ids directly, so the product path does
not build padded inverses; these helpers keep recipe code that does
portable.  Reference behaviour: recipes/recsys/ranking/schema/contracts.py,
sparse_features.py and input.py (the group-name rule and the knob grammar
are the reference's interface, kept for configuration files).
"""
from __future__ import annotations

from collections.abc import Iterable, Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np

from ..training.contracts import BatchFieldSpec, BatchSchema, TensorSpec


@dataclass(frozen=True)
class RankingBatch:
    sparse_features: Mapping[str, Any]
    side_info_features: Mapping[str, Any]
    labels: Mapping[str, Any]
    sample_weights: Mapping[str, Any] | None = None
    group_ids: Any | None = None
    valid_count: int | None = None


def build_ranking_batch_schema(sparse_groups: Sequence[str], *, side_info_groups: Sequence[str] = ("side_info",),
                               include_group_id: bool = True) -> BatchSchema:
    fields: dict[str, BatchFieldSpec] = {
        g: BatchFieldSpec(g, TensorSpec((None,), "int64"), is_sparse=True) for g in sparse_groups}
    for g in side_info_groups:
        fields[g] = BatchFieldSpec(g, TensorSpec((None, None), "float32"))
    fields["labels"] = BatchFieldSpec("labels", TensorSpec((None,), "int32"), is_label=True)
    if include_group_id:
        fields["group_id"] = BatchFieldSpec("group_id", TensorSpec((None,), "int64"))
    fields["samples_valid_count"] = BatchFieldSpec("samples_valid_count", TensorSpec((), "int32"))
    return BatchSchema(fields=fields)


# ------------------------------------------------------------- sparse groups
_DIM = "_dim_"


def parse_sparse_group_name(group_name: str) -> tuple[str, int]:
    if not isinstance(group_name, str) or not group_name:
        raise ValueError(f"sparse group name must be a non-empty string, got {group_name!r}")
    base, sep, dim = group_name.rpartition(_DIM)
    if not sep:
        raise ValueError(f"sparse group name must contain '{_DIM}<dimension>', got {group_name!r}")
    if not base:
        raise ValueError(f"sparse group base name must not be empty in {group_name!r}")
    try:
        d = int(dim)
    except ValueError as e:
        raise ValueError(f"invalid dimension in sparse group name {group_name!r}: {dim!r}") from e
    if d <= 0:
        raise ValueError(f"dimension in sparse group name {group_name!r} must be positive, got {d}")
    return base, d


def extract_sparse_groups_and_dimensions(sparse_id_groups) -> tuple[tuple[str, ...], dict[str, list[int]]]:
    if not isinstance(sparse_id_groups, (Mapping, tuple, list)):
        raise TypeError("sparse_id_groups must be a Mapping or Sequence of group names, "
                        f"got {type(sparse_id_groups).__name__}")
    names = tuple(sparse_id_groups)
    dims: dict[str, set[int]] = {}
    for n in names:
        b, d = parse_sparse_group_name(n)
        dims.setdefault(b, set()).add(d)
    return names, {b: sorted(v) for b, v in dims.items()}


def extract_sparse_base_names(sparse_groups: Iterable[str]) -> tuple[str, ...]:
    if not isinstance(sparse_groups, Iterable):
        raise TypeError("sparse_groups must be an Iterable")
    return tuple(sorted({parse_sparse_group_name(n)[0] for n in sparse_groups}))


def _positive(value: str, what: str) -> int:
    try:
        n = int(value)
    except ValueError as e:
        raise ValueError(f"{what} must be an integer, got {value!r}") from e
    if n <= 0:
        raise ValueError(f"{what} must be positive, got {n}")
    return n


def _group_counts(spec: str, sparse_groups: Iterable[str], what: str, default: int | None) -> dict[str, int]:
    if not isinstance(spec, str):
        raise TypeError(f"{what} must be a string")
    bases = extract_sparse_base_names(sparse_groups)
    out = {} if default is None else {b: default for b in bases}
    if not spec:
        return out
    if ":" not in spec:
        n = _positive(spec, what)
        return {b: n for b in bases}
    seen = set()
    for item in spec.split(","):
        parts = [x.strip() for x in item.split(":")]
        if len(parts) != 2:
            raise ValueError(f"{what} override must use name:count, got {item!r}")
        name, value = parts
        if name not in bases:
            raise ValueError(f"unknown sparse group {name!r}")
        if name in seen:
            raise ValueError(f"duplicate sparse group {name!r}")
        seen.add(name)
        out[name] = _positive(value, f"{what} for {name!r}")
    return out


def parse_sparse_workers(spec: str, sparse_groups: Iterable[str]) -> dict[str, int]:
    return _group_counts(spec, sparse_groups, "sparse worker count", 1)


def parse_sparse_thread_budgets(spec: str, sparse_groups: Iterable[str]) -> dict[str, int]:
    """Explicit per-group thread budgets; groups not named keep their default (absent from the result)."""
    return _group_counts(spec, sparse_groups, "sparse thread budget", None)


def build_sparse_group_feature_widths(categorical_feature_groups: Mapping[str, Sequence[str]],
                                      feature_lengths: Mapping[str, int],
                                      sparse_groups: Sequence[str]) -> dict[str, tuple[int, int]]:
    """group -> (number of features, widest feature length)."""
    if not isinstance(categorical_feature_groups, Mapping):
        raise TypeError("categorical_feature_groups must be a Mapping")
    out = {}
    for g in sparse_groups:
        if g not in categorical_feature_groups:
            raise KeyError(f"sparse group {g!r} is absent from the model's feature groups")
        feats = tuple(categorical_feature_groups[g])
        if not feats:
            raise ValueError(f"sparse group {g!r} must contain at least one feature")
        missing = [f for f in feats if f not in feature_lengths]
        if missing:
            raise KeyError(f"sparse group {g!r} has unknown feature lengths: {missing}")
        lens = tuple(int(feature_lengths[f]) for f in feats)
        if any(n <= 0 for n in lens):
            raise ValueError(f"sparse group {g!r} has invalid feature lengths: {lens}")
        out[g] = (len(feats), max(lens))
    return out


# ------------------------------------------------------------- padded inverse
def _host(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def validate_inverse_range(inverse, pad_index: int, group: str) -> None:
    v = _host(inverse).reshape(-1)
    if v.size == 0:
        raise ValueError(f"sparse inverse for group {group!r} has no slots")
    lo, hi = int(v.min()), int(v.max())
    if lo < 0 or hi > pad_index:
        raise IndexError(f"sparse inverse for group {group!r} is outside [0, {pad_index}]: "
                         f"minimum={lo}, maximum={hi}")


def materialize_padded_inverse(flat_values, nested_splits: Sequence[Any] | None, global_shape: tuple[int, ...] | None,
                               *, pad_index: int, batch_size: int, target_widths: tuple[int, ...], group: str,
                               output_dtype=np.int32, audit: bool = False) -> np.ndarray:
    dtype = np.dtype(output_dtype)
    if audit:
        if batch_size <= 0:
            raise ValueError(f"batch_size must be positive, got {batch_size}")
        if not target_widths or any(w <= 0 for w in target_widths):
            raise ValueError(f"target_widths must be positive, got {target_widths}")
        if dtype.kind not in "iu":
            raise TypeError(f"inverse dtype must be integral, got {dtype}")
        if not 0 <= pad_index <= int(np.iinfo(dtype).max):
            raise ValueError(f"pad_index {pad_index} does not fit {dtype}")
    flat = _host(flat_values)
    out = np.full((batch_size, *target_widths), pad_index, dtype=dtype)
    if not nested_splits:  # a dense prefix matrix
        widths = tuple(int(w) for w in flat.shape[1:])
        if audit:
            if flat.shape[0] != batch_size:
                raise ValueError(f"sparse inverse for group {group!r} has {flat.shape[0]} rows, expected {batch_size}")
            if len(widths) != len(target_widths) or any(a > t for a, t in zip(widths, target_widths)):
                raise ValueError(f"sparse inverse widths {widths} do not fit {target_widths} for group {group!r}")
            validate_inverse_range(flat, pad_index, group)
        out[(slice(None),) + tuple(slice(0, w) for w in widths)] = flat.astype(dtype, copy=False)
        return out
    if audit:
        if not global_shape or len(global_shape) != len(nested_splits) + 1:
            raise ValueError(f"ragged inverse for group {group!r} requires global_shape")
        if len(global_shape) - 1 != len(target_widths):
            raise ValueError(f"ragged inverse metadata rank differs from the target widths for group {group!r}")
        validate_inverse_range(flat, pad_index, group)
    splits = [_host(s).astype(np.int64).reshape(-1) for s in nested_splits]
    if len(splits) != len(target_widths) or splits[0].size != batch_size + 1:
        raise ValueError(f"ragged inverse shape mismatch for group {group!r}")
    # level by level: the flat position of every child in the padded output, and whether it fits
    pos = np.arange(batch_size, dtype=np.int64)
    ok = np.ones(batch_size, dtype=bool)
    for level, (sp, width) in enumerate(zip(splits, target_widths)):
        children = splits[level + 1].size - 1 if level + 1 < len(splits) else flat.size
        if sp.size != pos.size + 1 or sp[0] != 0 or sp[-1] != children or np.any(np.diff(sp) < 0):
            raise ValueError(f"invalid ragged inverse offsets for group {group!r} at level {level}")
        lens = np.diff(sp)
        parent = np.repeat(np.arange(pos.size), lens)
        local = np.arange(children) - sp[parent]
        ok = ok[parent] & (local < width)
        pos = pos[parent] * width + local
    out.reshape(-1)[pos[ok]] = flat.reshape(-1)[ok].astype(dtype, copy=False)
    return out


__all__ = ["RankingBatch", "build_ranking_batch_schema", "build_sparse_group_feature_widths",
           "extract_sparse_base_names", "extract_sparse_groups_and_dimensions", "materialize_padded_inverse",
           "parse_sparse_group_name", "parse_sparse_thread_budgets", "parse_sparse_workers",
           "validate_inverse_range"]
