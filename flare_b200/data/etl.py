"""Feature ETL for the offline production pipeline (native kernels + NumPy references).

``RecordScanner`` parses production log records (TAB-separated columns; the
feature column holds ``code\\x03value`` items separated by ``\\x02``, list
values comma separated) straight into NumPy buffers with the native scanner
(``csrc/etl.cpp``).  The encoders turn raw values into model inputs: hash
buckets, FNV-1a hashes of lists or (seed, value) pairs, bucketized or
fixed-width dense values, slot-packed 64-bit feature ids and list
intersections.  Missing values use the null sentinel -3.  Every native
function has a NumPy reference here (the numerics oracle of the tests).

Reference behaviour: src/flare/data/pipeline/production/processing/native/
_scan.pyx:73 (scanner) and builder/encoding/{sparse_id.py:206-290, dense.py:
30-45}, builder/cross/fea_ops.py:63-94 (encoders).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

NULL = -3
FNV_OFFSET = 14695981039346656037
FNV_PRIME = 1099511628211
M64 = (1 << 64) - 1


def _etl():
    from .._native import native

    return native().etl


@dataclass(frozen=True)
class FieldSpec:
    code: int
    length: int = 1
    is_float: bool = False


class RecordScanner:
    """Parse record bytes into per-field buffers (int64 or float64, [rows, length]) + validity."""

    def __init__(self, fields: list[FieldSpec], *, num_columns: int, feature_column: int | None = None):
        self.fields = list(fields)
        self.num_columns = num_columns
        self.feature_column = num_columns - 1 if feature_column is None else feature_column
        self.plan = {f.code: (i, f.length, f.is_float) for i, f in enumerate(self.fields)}

    def scan(self, data: bytes, max_rows: int) -> tuple[dict[int, np.ndarray], dict[int, np.ndarray], int]:
        bufs = [np.full((max_rows, f.length), NULL, dtype=np.float64 if f.is_float else np.int64)
                for f in self.fields]
        valid = [np.zeros(max_rows, dtype=np.uint8) for _ in self.fields]
        (rows,) = _etl().scan_records(data, self.num_columns, self.feature_column, self.plan, bufs, valid)
        return ({f.code: b[:rows] for f, b in zip(self.fields, bufs)},
                {f.code: v[:rows] for f, v in zip(self.fields, valid)}, rows)

    def scan_reference(self, data: bytes, max_rows: int):
        bufs = {f.code: np.full((max_rows, f.length), NULL, dtype=np.float64 if f.is_float else np.int64)
                for f in self.fields}
        valid = {f.code: np.zeros(max_rows, dtype=np.uint8) for f in self.fields}
        spec = {f.code: f for f in self.fields}
        rows = 0
        for line in data.split(b"\n"):
            if not line:
                continue
            cols = line.split(b"\t")
            if len(cols) > self.feature_column:
                for item in cols[self.feature_column].split(b"\x02"):
                    if b"\x03" not in item:
                        continue
                    code, val = item.split(b"\x03", 1)
                    try:
                        c = int(code)
                    except ValueError:
                        continue
                    if c not in spec:
                        continue
                    f = spec[c]
                    parts = val.split(b",") if f.length > 1 else [val]
                    for k, part in enumerate(parts[:f.length]):
                        try:
                            bufs[c][rows, k] = float(part) if f.is_float else int(float(part))
                        except ValueError:
                            bufs[c][rows, k] = NULL
                    valid[c][rows] = 1
            rows += 1
        return ({c: b[:rows] for c, b in bufs.items()}, {c: v[:rows] for c, v in valid.items()}, rows)


# ---------------------------------------------------------------- encoders
def hash_bucket(values: np.ndarray, buckets: int, default_value: int = NULL) -> np.ndarray:
    return _etl().hash_bucket(np.ascontiguousarray(values, dtype=np.int64), int(buckets), int(default_value))


def hash_bucket_reference(values, buckets, default_value=NULL):
    v = np.asarray(values, dtype=np.int64)
    out = (v.astype(np.uint64) % np.uint64(buckets)).astype(np.int64)
    out[(v == default_value) | (v == NULL)] = NULL
    return out


def fnv1a_lists(values: np.ndarray, offsets: np.ndarray, buckets: int = 0) -> np.ndarray:
    return _etl().fnv1a_lists(np.ascontiguousarray(values, dtype=np.int64),
                              np.ascontiguousarray(offsets, dtype=np.int64), int(buckets))


def fnv1a_lists_reference(values, offsets, buckets=0):
    out = []
    for i in range(len(offsets) - 1):
        h = FNV_OFFSET
        for v in values[offsets[i]:offsets[i + 1]]:
            h = ((h ^ (int(v) & M64)) * FNV_PRIME) & M64
        out.append(h % buckets if buckets else h)
    return np.array(out, dtype=np.uint64)


def fnv1a_seeded(values: np.ndarray, seed: int) -> np.ndarray:
    return _etl().fnv1a_seeded(np.ascontiguousarray(values, dtype=np.int64), int(seed))


def fnv1a_seeded_reference(values, seed):
    def feed(h, x, zero_byte):
        if x == 0 and zero_byte:
            return (h * FNV_PRIME) & M64
        while x > 0:
            h = ((h ^ (x & 0xFF)) * FNV_PRIME) & M64
            x >>= 8
        return h

    hs = feed(FNV_OFFSET, int(seed), False)
    return np.array([hs if int(v) < 0 else feed(hs, int(v), True) for v in values], dtype=np.uint64)


def bucketize(values: np.ndarray, bounds: np.ndarray, default_value: float = NULL) -> np.ndarray:
    return _etl().bucketize(np.ascontiguousarray(values, dtype=np.float32),
                            np.ascontiguousarray(np.sort(bounds), dtype=np.float32), float(default_value))


def bucketize_reference(values, bounds, default_value=NULL):
    v = np.asarray(values, dtype=np.float32)
    out = np.searchsorted(np.sort(np.asarray(bounds, dtype=np.float32)), v, side="left").astype(np.int32)
    out[(v == np.float32(NULL)) | (v == np.float32(default_value))] = NULL
    return out


def fixed_width(values: np.ndarray, width: float, default_value: float = NULL) -> np.ndarray:
    return _etl().fixed_width(np.ascontiguousarray(values, dtype=np.float32), float(width), float(default_value))


def pack_fids(values: np.ndarray, slot: int) -> np.ndarray:
    return _etl().pack_fids(np.ascontiguousarray(values, dtype=np.int64), int(slot))


def pack_fids_reference(values, slot):
    v = np.asarray(values, dtype=np.int64).astype(np.uint64) & np.uint64((1 << 48) - 1)
    return (v | np.uint64(slot << 48)).astype(np.int64)


def intersect_lists(a, oa, b, ob) -> np.ndarray:
    c = lambda x: np.ascontiguousarray(x, dtype=np.int64)  # noqa: E731
    return _etl().intersect_lists(c(a), c(oa), c(b), c(ob))


def intersect_lists_reference(a, oa, b, ob):
    out = []
    for i in range(len(oa) - 1):
        xs = [x for x in a[oa[i]:oa[i + 1]] if x != NULL]
        ys = list(b[ob[i]:ob[i + 1]])
        out.append(sum(1 for x in xs for y in ys if x == y))
    return np.array(out, dtype=np.int32)


__all__ = ["FieldSpec", "NULL", "RecordScanner", "bucketize", "fixed_width", "fnv1a_lists", "fnv1a_seeded",
           "hash_bucket", "intersect_lists", "pack_fids"]
