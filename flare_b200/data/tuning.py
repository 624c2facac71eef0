"""Memory-valid batch sizing for the feature-production workers.

``estimate_row_bytes(schema)`` estimates the in-memory bytes of one encoded
row from its Arrow schema (fixed-width values at their width, lists at an
assumed length plus offsets, strings and binaries at an assumed length).
``choose_encoded_batch`` picks the encoded batch target for a worker: wide
rows (>= 32 KiB) start at 256 MiB, narrower ones at 128 MiB, and an
automatic choice steps down (to 64 MiB) until the worker's peak -- the
decoded source batch, the encoded batch and the Parquet writer's buffers,
about four batches in flight -- fits in 90 % of its memory; a size supplied
by the caller is kept, or refused when it does not fit.

Reference behaviour: the schema-aware CPU profile of recipes/recsys/data/
ray_tuning.py:57-125 and the worker-memory planner it calls.
"""
from __future__ import annotations

from dataclasses import dataclass

import pyarrow as pa

MIB = 1024 * 1024
WIDE_ROW_BYTES = 32 * 1024
LIST_LENGTH = 16          # assumed elements of a list value
STRING_BYTES = 32         # assumed bytes of a string / binary value
BATCHES_IN_FLIGHT = 4     # decoded + encoded + writer buffers
MEMORY_FRACTION = 0.9


def _type_bytes(t: pa.DataType) -> int:
    if pa.types.is_list(t) or pa.types.is_large_list(t):
        return 4 + LIST_LENGTH * _type_bytes(t.value_type)
    if pa.types.is_fixed_size_list(t):
        return t.list_size * _type_bytes(t.value_type)
    if pa.types.is_struct(t):
        return sum(_type_bytes(t.field(i).type) for i in range(t.num_fields))
    if pa.types.is_string(t) or pa.types.is_binary(t) or pa.types.is_large_string(t):
        return 4 + STRING_BYTES
    if pa.types.is_boolean(t):
        return 1
    try:
        return max(1, t.bit_width // 8)
    except ValueError:
        return 8


def estimate_row_bytes(schema: pa.Schema) -> int:
    return max(1, sum(_type_bytes(f.type) + 1 for f in schema))  # + validity


@dataclass(frozen=True)
class EncodedBatchTarget:
    batch_bytes: int
    row_bytes: int
    rows_per_batch: int
    peak_bytes: int


def choose_encoded_batch(schema: pa.Schema, *, worker_memory_bytes: int,
                         supplied: int | None = None) -> EncodedBatchTarget:
    row = estimate_row_bytes(schema)
    if supplied is not None:
        options = (int(supplied),)
    elif row >= WIDE_ROW_BYTES:
        options = (256 * MIB, 128 * MIB, 64 * MIB)
    else:
        options = (128 * MIB, 64 * MIB)
    limit = int(worker_memory_bytes * MEMORY_FRACTION)
    for b in options:
        peak = BATCHES_IN_FLIGHT * b
        if peak <= limit:
            return EncodedBatchTarget(b, row, max(1, b // row), peak)
    raise ValueError(f"no encoded batch size fits a worker of {worker_memory_bytes / MIB:.0f} MiB "
                     f"(tried {[o // MIB for o in options]} MiB)")


__all__ = ["EncodedBatchTarget", "MIB", "choose_encoded_batch", "estimate_row_bytes"]
