"""Row operations on routed ragged batches that keep their routing metadata.

A ``RoutedRagged`` is a ragged tensor (flat values + nested int32 row splits,
NumPy or torch, host or device) plus the metadata that lets a receiver put
its rows back in global order: ``origin`` (global row index of every row, -1
for padding), ``global_rows`` and ``source_step``.  ``concatenate`` merges
batches of the same step (splits re-based, origins concatenated), ``take``
slices rows, ``pad`` appends copies of the last row marked as padding
(origin -1), so a fixed-shape consumer (a CUDA graph) sees full batches while
the valid rows stay identifiable.  Reference behaviour:
src/flare/runtime/fluxway/transport.py:100-260 (TransportTensorOperations).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


def _is_torch(x) -> bool:
    return isinstance(x, torch.Tensor)


def _cat(xs):
    return torch.cat(xs) if _is_torch(xs[0]) else np.concatenate(xs)


def _cumsum0(lengths):
    if _is_torch(lengths):
        z = torch.zeros(1, dtype=torch.int32, device=lengths.device)
        return torch.cat([z, torch.cumsum(lengths, 0).to(torch.int32)])
    return np.concatenate([np.zeros(1, np.int32), np.cumsum(lengths).astype(np.int32)])


@dataclass(frozen=True)
class RoutedRagged:
    flat_values: object
    splits: tuple          # nested row splits, outermost first (int32, start at 0)
    origin: object         # int64 global row index per outer row, -1 = padding
    global_rows: int
    source_step: int = 0

    def __post_init__(self) -> None:
        if not self.splits:
            raise ValueError("a ragged batch needs at least one split level")
        inner = len(self.flat_values)
        for s in reversed(self.splits):
            if int(s[0]) != 0 or int(s[-1]) != inner:
                raise ValueError("row splits must start at 0 and end at the inner length")
            inner = len(s) - 1
        if len(self.origin) != self.rows:
            raise ValueError("origin must have one entry per row")

    @property
    def rows(self) -> int:
        return len(self.splits[0]) - 1

    def valid_rows(self) -> int:
        o = self.origin
        return int((o >= 0).sum())


def concatenate(parts: list[RoutedRagged]) -> RoutedRagged:
    if not parts:
        raise ValueError("nothing to concatenate")
    if len(parts) == 1:
        return parts[0]
    f = parts[0]
    if any(p.global_rows != f.global_rows for p in parts):
        raise ValueError("global_rows conflict")
    if any(p.source_step != f.source_step for p in parts):
        raise ValueError("batches of different source steps")
    if any(len(p.splits) != len(f.splits) for p in parts):
        raise ValueError("different nesting levels")
    splits = []
    for lvl in range(len(f.splits)):
        lengths = _cat([p.splits[lvl][1:] - p.splits[lvl][:-1] for p in parts])
        splits.append(_cumsum0(lengths))
    return RoutedRagged(_cat([p.flat_values for p in parts]), tuple(splits), _cat([p.origin for p in parts]),
                        f.global_rows, f.source_step)


def take(x: RoutedRagged, start: int, count: int) -> RoutedRagged:
    """Rows [start, start + count)."""
    if start < 0 or count < 0 or start + count > x.rows:
        raise ValueError(f"rows [{start}, {start + count}) outside [0, {x.rows})")
    lo, hi = start, start + count
    splits = []
    for s in x.splits:
        a, b = int(s[lo]), int(s[hi])
        splits.append(s[lo:hi + 1] - s[lo])
        lo, hi = a, b
    return RoutedRagged(x.flat_values[lo:hi], tuple(splits), x.origin[start:start + count], x.global_rows,
                        x.source_step)


def pad(x: RoutedRagged, count: int) -> RoutedRagged:
    """Append ``count`` copies of the last row, marked as padding (origin -1)."""
    if count < 0:
        raise ValueError("padding count must be non-negative")
    if count == 0:
        return x
    if x.rows == 0:
        raise ValueError("cannot pad an empty batch")
    last = take(x, x.rows - 1, 1)
    filler = [RoutedRagged(last.flat_values, last.splits, last.origin * 0 - 1, x.global_rows, x.source_step)]
    return concatenate([x] + filler * count)


__all__ = ["RoutedRagged", "concatenate", "pad", "take"]
