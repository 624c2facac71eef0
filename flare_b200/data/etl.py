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


class ArrowRowParser:
    """Parse an Arrow string column of records (one record per row) without per-row Python objects.

    ``fixed``: code -> (length, is_float) fixed-width outputs [rows, length];
    ``lists``: code -> is_float variable-length outputs (values, int64 offsets [rows+1]);
    ``categories``: code -> (vocabulary {token: index}, default index) -> int32 [rows];
    ``direct``: name -> TAB column parsed as int64; ``metadata``: name -> (TAB column,
    {string: id}, default id) -> int32.  Missing values are -3 (``NULL``).
    Reference behaviour: src/flare/data/pipeline/production/builder/_fast_parse.pyx:87-350.
    """

    def __init__(self, *, feature_column: int, fixed=None, lists=None, categories=None, direct=None,
                 metadata=None):
        self.feature_column = feature_column
        self.fixed = dict(fixed or {})
        self.lists = dict(lists or {})
        self.categories = {c: (dict(v), int(d)) for c, (v, d) in (categories or {}).items()}
        self.direct = dict(direct or {})
        self.metadata = {n: (c, dict(t), int(d)) for n, (c, t, d) in (metadata or {}).items()}
        both = set(self.fixed) & set(self.lists) | set(self.fixed) & set(self.categories) | \
            set(self.lists) & set(self.categories)
        if both:
            raise ValueError(f"feature codes with two output kinds: {sorted(both)}")

    @staticmethod
    def _buffers(column):
        import pyarrow as pa

        if isinstance(column, pa.ChunkedArray):
            column = column.combine_chunks()
        if pa.types.is_large_string(column.type) or pa.types.is_large_binary(column.type):
            odt = np.int64
        elif pa.types.is_string(column.type) or pa.types.is_binary(column.type):
            odt = np.int32
        else:
            raise TypeError(f"expected a string column, got {column.type}")
        _, obuf, dbuf = column.buffers()
        n = len(column)
        offs = np.frombuffer(obuf, dtype=odt, count=column.offset + n + 1)[column.offset:].astype(np.int64)
        data = np.frombuffer(dbuf, dtype=np.uint8) if dbuf is not None else np.zeros(1, np.uint8)
        return data, offs, n

    def parse(self, column, *, list_capacity: int | None = None) -> dict:
        data, offs, n = self._buffers(column)
        cap = list_capacity or max(16, int(offs[-1] - offs[0]) // 2 + 16)
        plan, out = {}, {"fixed": {}, "lists": {}, "categories": {}, "direct": {}, "metadata": {}, "valid": {}}
        for code, (length, is_float) in self.fixed.items():
            buf = np.empty((n, length), dtype=np.float64 if is_float else np.int64)
            val = np.empty(n, dtype=np.uint8)
            plan[code] = (0, length, bool(is_float), buf, None, val)
            out["fixed"][code], out["valid"][code] = buf, val
        for code, is_float in self.lists.items():
            vals = np.empty(cap, dtype=np.float64 if is_float else np.int64)
            lo = np.empty(n + 1, dtype=np.int64)
            val = np.empty(n, dtype=np.uint8)
            plan[code] = (1, 0, bool(is_float), vals, lo, val)
            out["lists"][code], out["valid"][code] = (vals, lo), val
        cats = {}
        for code, (vocab, dflt) in self.categories.items():
            buf = np.empty(n, dtype=np.int32)
            val = np.empty(n, dtype=np.uint8)
            plan[code] = (2, 1, False, buf, None, val)
            cats[code] = ({k.encode() if isinstance(k, str) else k: v for k, v in vocab.items()}, dflt)
            out["categories"][code], out["valid"][code] = buf, val
        direct = []
        for name, col in self.direct.items():
            buf = np.empty(n, dtype=np.int64)
            direct.append((col, buf, None))
            out["direct"][name] = buf
        meta = []
        for name, (col, table, dflt) in self.metadata.items():
            buf = np.empty(n, dtype=np.int32)
            meta.append((col, {k.encode() if isinstance(k, str) else k: v for k, v in table.items()}, dflt, buf))
            out["metadata"][name] = buf
        _, counts = _etl().parse_rows(data, offs, n, self.feature_column, plan, cats, direct, meta)
        for code, used in counts.items():
            vals, lo = out["lists"][code]
            out["lists"][code] = (vals[:used], lo)
        return out

    def parse_reference(self, lines: list[str]) -> dict:
        """Pure-Python restatement (the oracle of the tests)."""
        n = len(lines)
        res = {"fixed": {c: np.full((n, ln), NULL, dtype=np.float64 if f else np.int64)
                         for c, (ln, f) in self.fixed.items()},
               "lists": {c: [[] for _ in range(n)] for c in self.lists},
               "categories": {c: np.full(n, NULL, dtype=np.int32) for c in self.categories},
               "direct": {k: np.full(n, NULL, dtype=np.int64) for k in self.direct},
               "metadata": {k: np.full(n, d, dtype=np.int32) for k, (_, _, d) in self.metadata.items()}}

        def num(tok, is_float):
            try:
                return float(tok) if is_float else int(float(tok))
            except ValueError:
                return NULL

        for r, line in enumerate(lines):
            cols = line.rstrip("\n").split("\t")
            for k, col in self.direct.items():
                if col < len(cols) and cols[col]:
                    res["direct"][k][r] = num(cols[col], False)
            for k, (col, table, d) in self.metadata.items():
                if col < len(cols):
                    res["metadata"][k][r] = table.get(cols[col], d)
            if self.feature_column >= len(cols):
                continue
            for item in cols[self.feature_column].split("\x02"):
                if "\x03" not in item:
                    continue
                code_s, val = item.split("\x03", 1)
                code = num(code_s, False)
                if code in self.fixed:
                    ln, f = self.fixed[code]
                    parts = val.split(",") if ln > 1 else [val]
                    for j, tok in enumerate(parts[:ln]):
                        res["fixed"][code][r, j] = num(tok, f)
                elif code in self.lists:
                    res["lists"][code][r] = [num(t, self.lists[code]) for t in val.split(",") if t != ""]
                elif code in self.categories:
                    vocab, d = self.categories[code]
                    res["categories"][code][r] = vocab.get(val, d)
        return res


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


__all__ = ["ArrowRowParser", "FieldSpec", "NULL", "RecordScanner", "bucketize", "fixed_width", "fnv1a_lists", "fnv1a_seeded",
           "hash_bucket", "intersect_lists", "pack_fids"]
