"""Avro codec (CPU): zig-zag varints against the specification's examples, container round trips
(null and deflate codecs, nested records, unions, arrays, maps, enums, fixed, named references)."""
import io

import pytest

from flare_b200.data.avro import (ContainerReader, Schema, _read_long, _write_long, container_bytes, decode,
                                  encode, read_container)


@pytest.mark.parametrize("v,enc", [(0, b"\x00"), (-1, b"\x01"), (1, b"\x02"), (-2, b"\x03"), (2, b"\x04"),
                                   (-64, b"\x7f"), (64, b"\x80\x01")])
def test_zigzag_examples_of_the_specification(v, enc):
    out = io.BytesIO()
    _write_long(out, v)
    assert out.getvalue() == enc
    assert _read_long(io.BytesIO(enc)) == v


SCHEMA = {
    "type": "record", "name": "entry", "namespace": "t",
    "fields": [
        {"name": "status", "type": "int"},
        {"name": "id", "type": ["null", "long"], "default": None},
        {"name": "score", "type": "double"},
        {"name": "ok", "type": "boolean"},
        {"name": "kind", "type": {"type": "enum", "name": "Kind", "symbols": ["DATA", "DELETES"]}},
        {"name": "hash", "type": {"type": "fixed", "name": "Hash", "size": 4}},
        {"name": "file", "type": {"type": "record", "name": "file", "fields": [
            {"name": "path", "type": "string"},
            {"name": "sizes", "type": {"type": "map", "values": "long"}},
            {"name": "bounds", "type": {"type": "array", "items": "bytes"}},
            {"name": "ts", "type": {"type": "long", "logicalType": "timestamp-micros"}},
        ]}},
        {"name": "other", "type": ["null", "file"], "default": None},
    ],
}


def _rec(i):
    f = {"path": f"s3://b/d/{i}.parquet", "sizes": {"1": i, "2": 2 * i}, "bounds": [b"a", bytes([i % 256])],
         "ts": 1_700_000_000_000_000 + i}
    return {"status": i % 3, "id": None if i % 2 else -(i << 40), "score": i / 7.0, "ok": bool(i % 2),
            "kind": "DELETES" if i % 5 == 0 else "DATA", "hash": bytes([1, 2, 3, i % 256]), "file": f,
            "other": f if i % 3 == 0 else None}


@pytest.mark.parametrize("codec", ["null", "deflate"])
def test_container_round_trip(codec):
    recs = [_rec(i) for i in range(2500)]
    data = container_bytes(SCHEMA, recs, codec=codec, metadata={"format-version": "2"}, block_records=700)
    back, meta = read_container(data)
    assert back == recs
    assert meta["format-version"] == b"2" and meta["avro.codec"] == codec.encode()
    assert ContainerReader(data).schema_json == SCHEMA


def test_defaults_unions_and_errors():
    s = Schema(SCHEMA)
    r = _rec(3)
    del r["id"]  # defaulted field
    out = io.BytesIO()
    encode(s.root, r, out)
    got = decode(s.root, io.BytesIO(out.getvalue()))
    assert got["id"] is None
    with pytest.raises(ValueError, match="misses field"):
        encode(s.root, {"status": 1}, io.BytesIO())
    with pytest.raises(ValueError, match="no union branch"):
        encode(Schema(["null", "long"]).root, "x", io.BytesIO())
    with pytest.raises(ValueError, match="not an Avro"):
        ContainerReader(b"nope")
    with pytest.raises(ValueError, match="unknown Avro type"):
        Schema({"type": "record", "name": "r", "fields": [{"name": "a", "type": "missing"}]})


def test_negative_block_counts_are_read():
    # an array written as one block with a negative count followed by its byte size
    out = io.BytesIO()
    items = io.BytesIO()
    for v in (5, 6, 7):
        _write_long(items, v)
    _write_long(out, -3)
    _write_long(out, len(items.getvalue()))
    out.write(items.getvalue())
    _write_long(out, 0)
    assert decode(Schema({"type": "array", "items": "long"}).root, io.BytesIO(out.getvalue())) == [5, 6, 7]
