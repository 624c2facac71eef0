"""Avro object container files, read and written without an Avro library.

Binary encoding (Avro 1.x specification): ``null`` is empty; ``boolean`` one
byte; ``int`` / ``long`` zig-zag varints; ``float`` / ``double`` little-endian
IEEE; ``bytes`` / ``string`` a long length then the bytes; ``fixed`` its size
in bytes; ``enum`` the symbol's index; ``array`` / ``map`` blocks of (count,
items) ending with a zero count (a negative count is followed by the block's
byte size); ``union`` the branch index then the value; ``record`` its fields
in order.  A container file is the magic ``Obj\\x01``, a metadata map
(``avro.schema`` JSON, ``avro.codec``), a 16-byte sync marker, then blocks of
(object count, byte size, data, sync marker).  Codecs: ``null`` and
``deflate`` (raw DEFLATE, RFC 1951).

Values map to Python as: record -> dict, array -> list, map -> dict, union
-> the branch's value (writing picks the first branch that accepts it),
enum -> symbol string, bytes / fixed -> bytes.  Named types may be referred
to by name after their definition; field aliases and default values are read
from the writer's schema only (no reader-schema resolution).  Used by the
Iceberg manifests (``data/iceberg.py``).
"""
from __future__ import annotations

import io
import json
import os
import struct
import zlib
from collections.abc import Iterable, Iterator
from typing import Any, BinaryIO

MAGIC = b"Obj\x01"
SYNC_SIZE = 16


# ------------------------------------------------------------------ primitives
def _write_long(out: BinaryIO, v: int) -> None:
    v = (v << 1) ^ (v >> 63)  # zig-zag
    v &= (1 << 64) - 1
    buf = bytearray()
    while v & ~0x7F:
        buf.append((v & 0x7F) | 0x80)
        v >>= 7
    buf.append(v)
    out.write(bytes(buf))


def _read_long(inp: BinaryIO) -> int:
    shift = n = 0
    while True:
        b = inp.read(1)
        if not b:
            raise EOFError("truncated Avro varint")
        c = b[0]
        n |= (c & 0x7F) << shift
        if not c & 0x80:
            break
        shift += 7
    return (n >> 1) ^ -(n & 1)


def _write_bytes(out: BinaryIO, b: bytes) -> None:
    _write_long(out, len(b))
    out.write(b)


def _read_bytes(inp: BinaryIO) -> bytes:
    n = _read_long(inp)
    if n < 0:
        raise ValueError("negative Avro byte length")
    b = inp.read(n)
    if len(b) != n:
        raise EOFError("truncated Avro bytes")
    return b


_PRIMS = ("null", "boolean", "int", "long", "float", "double", "bytes", "string")


class Schema:
    """A parsed schema with its named types resolved."""

    def __init__(self, schema: Any):
        self.named: dict[str, Any] = {}
        self.root = self._parse(schema, None)

    def _full(self, name: str, ns: str | None) -> str:
        return name if "." in name or not ns else f"{ns}.{name}"

    def _parse(self, s: Any, ns: str | None) -> Any:
        if isinstance(s, str):
            if s in _PRIMS:
                return s
            for key in (s, self._full(s, ns)):
                if key in self.named:
                    return self.named[key]
            raise ValueError(f"unknown Avro type {s!r}")
        if isinstance(s, list):
            return {"type": "union", "branches": [self._parse(b, ns) for b in s]}
        if not isinstance(s, dict):
            raise ValueError(f"bad Avro schema node {s!r}")
        t = s["type"]
        if isinstance(t, (dict, list)) or (isinstance(t, str) and t not in
                                           ("record", "error", "enum", "fixed", "array", "map") and t not in _PRIMS):
            return self._parse(t, ns)
        if t in _PRIMS:
            return t  # {"type": "long", "logicalType": ...}: the logical type is carried as its base type
        if t in ("record", "error", "enum", "fixed"):
            ns2 = s.get("namespace", ns)
            full = self._full(s["name"], ns2)
            node: dict[str, Any] = {"type": t, "name": full, "schema": s}
            self.named[full] = node
            self.named.setdefault(s["name"], node)
            if t in ("record", "error"):
                node["fields"] = [(f["name"], self._parse(f["type"], ns2), f) for f in s["fields"]]
            elif t == "enum":
                node["symbols"] = list(s["symbols"])
            else:
                node["size"] = int(s["size"])
            return node
        if t == "array":
            return {"type": "array", "items": self._parse(s["items"], ns)}
        if t == "map":
            return {"type": "map", "values": self._parse(s["values"], ns)}
        raise ValueError(f"unsupported Avro type {t!r}")


def _accepts(node: Any, v: Any) -> bool:
    t = node if isinstance(node, str) else node["type"]
    if t == "null":
        return v is None
    if t == "boolean":
        return isinstance(v, bool)
    if t in ("int", "long"):
        return isinstance(v, int) and not isinstance(v, bool)
    if t in ("float", "double"):
        return isinstance(v, (int, float)) and not isinstance(v, bool)
    if t == "string":
        return isinstance(v, str)
    if t in ("bytes", "fixed"):
        return isinstance(v, (bytes, bytearray))
    if t in ("record", "error", "map"):
        return isinstance(v, dict)
    if t == "array":
        return isinstance(v, (list, tuple))
    if t == "enum":
        return isinstance(v, str) and v in node["symbols"]
    return False


def encode(node: Any, v: Any, out: BinaryIO) -> None:
    t = node if isinstance(node, str) else node["type"]
    if t == "null":
        return
    if t == "boolean":
        out.write(b"\x01" if v else b"\x00")
    elif t in ("int", "long"):
        _write_long(out, int(v))
    elif t == "float":
        out.write(struct.pack("<f", float(v)))
    elif t == "double":
        out.write(struct.pack("<d", float(v)))
    elif t == "bytes":
        _write_bytes(out, bytes(v))
    elif t == "string":
        _write_bytes(out, v.encode("utf-8"))
    elif t == "fixed":
        if len(v) != node["size"]:
            raise ValueError(f"fixed {node['name']} needs {node['size']} bytes")
        out.write(bytes(v))
    elif t == "enum":
        _write_long(out, node["symbols"].index(v))
    elif t == "array":
        if v:
            _write_long(out, len(v))
            for x in v:
                encode(node["items"], x, out)
        _write_long(out, 0)
    elif t == "map":
        if v:
            _write_long(out, len(v))
            for k, x in v.items():
                _write_bytes(out, str(k).encode("utf-8"))
                encode(node["values"], x, out)
        _write_long(out, 0)
    elif t == "union":
        for i, b in enumerate(node["branches"]):
            if _accepts(b, v):
                _write_long(out, i)
                encode(b, v, out)
                return
        raise ValueError(f"no union branch accepts {v!r}")
    elif t in ("record", "error"):
        for name, fnode, fdef in node["fields"]:
            if name in v:
                val = v[name]
            elif "default" in fdef:
                val = fdef["default"]
            else:
                raise ValueError(f"record {node['name']} misses field {name!r}")
            encode(fnode, val, out)
    else:
        raise ValueError(f"cannot encode Avro type {t!r}")


def decode(node: Any, inp: BinaryIO) -> Any:
    t = node if isinstance(node, str) else node["type"]
    if t == "null":
        return None
    if t == "boolean":
        return inp.read(1) == b"\x01"
    if t in ("int", "long"):
        return _read_long(inp)
    if t == "float":
        return struct.unpack("<f", inp.read(4))[0]
    if t == "double":
        return struct.unpack("<d", inp.read(8))[0]
    if t == "bytes":
        return _read_bytes(inp)
    if t == "string":
        return _read_bytes(inp).decode("utf-8")
    if t == "fixed":
        return inp.read(node["size"])
    if t == "enum":
        return node["symbols"][_read_long(inp)]
    if t in ("array", "map"):
        out: Any = [] if t == "array" else {}
        while True:
            n = _read_long(inp)
            if n == 0:
                return out
            if n < 0:
                n = -n
                _read_long(inp)  # block byte size
            for _ in range(n):
                if t == "array":
                    out.append(decode(node["items"], inp))
                else:
                    k = _read_bytes(inp).decode("utf-8")
                    out[k] = decode(node["values"], inp)
    if t == "union":
        i = _read_long(inp)
        return decode(node["branches"][i], inp)
    if t in ("record", "error"):
        return {name: decode(fnode, inp) for name, fnode, _ in node["fields"]}
    raise ValueError(f"cannot decode Avro type {t!r}")


# ------------------------------------------------------------------ containers
_META = {"type": "map", "values": "bytes"}


def write_container(out: BinaryIO, schema: Any, records: Iterable[Any], *, codec: str = "deflate",
                    metadata: dict[str, str] | None = None, block_records: int = 1000) -> None:
    if codec not in ("null", "deflate"):
        raise ValueError(f"unsupported Avro codec {codec!r}")
    sch = Schema(schema)
    meta = {"avro.schema": json.dumps(schema).encode(), "avro.codec": codec.encode()}
    for k, v in (metadata or {}).items():
        meta[k] = v.encode() if isinstance(v, str) else bytes(v)
    sync = os.urandom(SYNC_SIZE)
    out.write(MAGIC)
    encode(_META, meta, out)
    out.write(sync)
    block, count = io.BytesIO(), 0

    def flush():
        nonlocal block, count
        if not count:
            return
        data = block.getvalue()
        if codec == "deflate":
            c = zlib.compressobj(6, zlib.DEFLATED, -15)
            data = c.compress(data) + c.flush()
        _write_long(out, count)
        _write_long(out, len(data))
        out.write(data)
        out.write(sync)
        block, count = io.BytesIO(), 0

    for r in records:
        encode(sch.root, r, block)
        count += 1
        if count >= block_records:
            flush()
    flush()


def container_bytes(schema: Any, records: Iterable[Any], **kw) -> bytes:
    buf = io.BytesIO()
    write_container(buf, schema, records, **kw)
    return buf.getvalue()


class ContainerReader:
    """Records of an Avro container (``metadata`` has the header's key/value map as bytes)."""

    def __init__(self, data: bytes | BinaryIO):
        self._inp = io.BytesIO(data) if isinstance(data, (bytes, bytearray)) else data
        if self._inp.read(4) != MAGIC:
            raise ValueError("not an Avro object container file")
        self.metadata: dict[str, bytes] = decode(_META, self._inp)
        self.schema_json = json.loads(self.metadata["avro.schema"].decode())
        self.codec = self.metadata.get("avro.codec", b"null").decode()
        if self.codec not in ("null", "deflate"):
            raise ValueError(f"unsupported Avro codec {self.codec!r}")
        self.schema = Schema(self.schema_json)
        self._sync = self._inp.read(SYNC_SIZE)

    def __iter__(self) -> Iterator[Any]:
        while True:
            head = self._inp.read(1)
            if not head:
                return
            self._inp.seek(-1, io.SEEK_CUR)
            count = _read_long(self._inp)
            size = _read_long(self._inp)
            data = self._inp.read(size)
            if self.codec == "deflate":
                data = zlib.decompress(data, -15)
            if self._inp.read(SYNC_SIZE) != self._sync:
                raise ValueError("Avro block sync marker mismatch")
            blk = io.BytesIO(data)
            for _ in range(count):
                yield decode(self.schema.root, blk)


def read_container(data: bytes) -> tuple[list[Any], dict[str, bytes]]:
    r = ContainerReader(data)
    return list(r), r.metadata


__all__ = ["ContainerReader", "Schema", "container_bytes", "decode", "encode", "read_container", "write_container"]
