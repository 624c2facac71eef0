"""Perfetto traces (protobuf ``Trace`` files) written and read without the perfetto package.

Only the part of the schema that slice timelines need: ``Trace.packet`` (1)
of ``TracePacket`` with ``timestamp`` (8), ``trusted_packet_sequence_id``
(10), ``track_event`` (11) and ``track_descriptor`` (60); ``TrackDescriptor``
with ``uuid`` (1), ``name`` (2), ``parent_uuid`` (5); ``TrackEvent`` with
``debug_annotations`` (4), ``type`` (9: slice begin 1, end 2, instant 3),
``track_uuid`` (11), ``name`` (23); ``DebugAnnotation`` with ``name`` (10)
and one of bool (2), uint (3), int (4), double (5), string (6).  These field
numbers are the published Perfetto schema, so the files open in the Perfetto
UI and traces from other Perfetto writers parse here.

``PerfettoWriter`` makes a track per (rank, lane) under a per-rank parent
track and records slices with integer / string / float annotations (the
phase tools key on ``step``).  ``parse_trace`` returns the slices as dicts
``{ts_ns, dur_ns, track, track_uuid, name, payload}`` with full ``/``-joined
track names, pairing begin / end per (track, name).

Reference counterpart: tools/validation/perfetto_trace.py (parser of the
Fluxway runtime's Perfetto traces, per-step statistics).
"""
from __future__ import annotations

import statistics
import struct
from collections import Counter, defaultdict
from pathlib import Path
from typing import Any

SLICE_BEGIN, SLICE_END, INSTANT = 1, 2, 3


# ------------------------------------------------------------------ wire format
def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1  # negative int64 values travel as their two's complement
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint(field << 3 | wire)


def _uint(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(int(v))


def _bytes(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _double(field: int, v: float) -> bytes:
    return _key(field, 1) + struct.pack("<d", float(v))


def _fields(buf: bytes):
    """(field number, wire type, value) of one message; length-delimited values as bytes."""
    i, n = 0, len(buf)
    while i < n:
        key, i = _read_varint(buf, i)
        field, wire = key >> 3, key & 7
        if wire == 0:
            v, i = _read_varint(buf, i)
        elif wire == 1:
            v = buf[i:i + 8]
            i += 8
        elif wire == 2:
            ln, i = _read_varint(buf, i)
            v = buf[i:i + ln]
            i += ln
        elif wire == 5:
            v = buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wire}")
        yield field, wire, v


def _read_varint(buf: bytes, i: int) -> tuple[int, int]:
    shift = v = 0
    while True:
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if not b & 0x80:
            return v, i
        shift += 7


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


# ---------------------------------------------------------------------- writer
def _annotation(name: str, value: Any) -> bytes:
    body = _bytes(10, name.encode())
    if isinstance(value, bool):
        body += _uint(2, 1 if value else 0)
    elif isinstance(value, int):
        body += _uint(4, value)
    elif isinstance(value, float):
        body += _double(5, value)
    else:
        body += _bytes(6, str(value).encode())
    return body


class PerfettoWriter:
    """Slices on named tracks, written as one Perfetto ``Trace`` file by ``save``."""

    SEQ = 1

    def __init__(self):
        self._packets: list[bytes] = []
        self._tracks: dict[tuple[str, ...], int] = {}
        self._next_uuid = 1000

    def track(self, *path: str) -> int:
        """uuid of the track ``path`` (parents created as needed), e.g. ``("rank:0", "compute")``."""
        path = tuple(path)
        if path in self._tracks:
            return self._tracks[path]
        parent = self.track(*path[:-1]) if len(path) > 1 else 0
        uuid = self._next_uuid
        self._next_uuid += 1
        desc = _uint(1, uuid) + _bytes(2, path[-1].encode()) + (_uint(5, parent) if parent else b"")
        self._packets.append(_uint(10, self.SEQ) + _bytes(60, desc))
        self._tracks[path] = uuid
        return uuid

    def _event(self, ts_ns: int, kind: int, track: int, name: str | None, args: dict | None) -> None:
        ev = _uint(9, kind) + _uint(11, track)
        if name is not None:
            ev += _bytes(23, name.encode())
        for k, v in (args or {}).items():
            ev += _bytes(4, _annotation(k, v))
        self._packets.append(_uint(8, int(ts_ns)) + _uint(10, self.SEQ) + _bytes(11, ev))

    def slice(self, track: tuple[str, ...], name: str, start_ns: int, end_ns: int, **args) -> None:
        if end_ns < start_ns:
            raise ValueError(f"slice {name!r} ends before it starts")
        uuid = self.track(*track)
        self._event(start_ns, SLICE_BEGIN, uuid, name, args)
        self._event(end_ns, SLICE_END, uuid, name, None)

    def instant(self, track: tuple[str, ...], name: str, ts_ns: int, **args) -> None:
        self._event(ts_ns, INSTANT, self.track(*track), name, args)

    def save(self, path: str | Path) -> Path:
        path = Path(path)
        path.write_bytes(b"".join(_bytes(1, p) for p in self._packets))
        return path


# ---------------------------------------------------------------------- reader
def _annotation_value(buf: bytes) -> tuple[str, Any]:
    name, value = "", None
    for f, w, v in _fields(buf):
        if f == 10:
            name = v.decode()
        elif f == 2:
            value = bool(v)
        elif f == 3:
            value = int(v)
        elif f == 4:
            value = _signed(int(v))
        elif f == 5:
            value = struct.unpack("<d", v)[0]
        elif f == 6:
            value = v.decode()
    return name, value


def parse_trace(path: str | Path) -> list[dict[str, Any]]:
    """Slices (and instants, with ``dur_ns`` 0) of a Perfetto trace file."""
    data = Path(path).read_bytes()
    names: dict[int, str] = {}
    parents: dict[int, int] = {}
    raw_events = []
    for f, _, pkt in _fields(data):
        if f != 1:
            continue
        ts, ev, desc = 0, None, None
        for pf, _, pv in _fields(pkt):
            if pf == 8:
                ts = int(pv)
            elif pf == 11:
                ev = pv
            elif pf == 60:
                desc = pv
        if desc is not None:
            uuid = parent = 0
            name = ""
            for df, _, dv in _fields(desc):
                if df == 1:
                    uuid = int(dv)
                elif df == 2:
                    name = dv.decode()
                elif df == 5:
                    parent = int(dv)
            names[uuid], parents[uuid] = name, parent
        if ev is not None:
            raw_events.append((ts, ev))

    def full(uuid: int) -> str:
        parts, seen = [], set()
        while uuid and uuid not in seen:
            seen.add(uuid)
            if names.get(uuid):
                parts.append(names[uuid])
            uuid = parents.get(uuid, 0)
        return "/".join(reversed(parts))

    out, open_slices = [], defaultdict(list)
    for ts, ev in raw_events:
        kind, track, name, payload = 0, 0, None, {}
        for ef, _, evv in _fields(ev):
            if ef == 9:
                kind = int(evv)
            elif ef == 11:
                track = int(evv)
            elif ef == 23:
                name = evv.decode()
            elif ef == 4:
                k, v = _annotation_value(evv)
                payload[k] = v
        if kind == SLICE_BEGIN:
            open_slices[track].append((ts, name, payload))
        elif kind == SLICE_END:
            if not open_slices[track]:
                raise ValueError(f"slice end without a begin on track {full(track)!r}")
            t0, bname, bpayload = open_slices[track].pop()
            if ts < t0:
                raise ValueError(f"slice {bname!r} has a negative duration")
            out.append({"ts_ns": t0, "dur_ns": ts - t0, "track": full(track), "track_uuid": track,
                        "name": bname, "payload": bpayload})
        else:
            out.append({"ts_ns": ts, "dur_ns": 0, "track": full(track), "track_uuid": track, "name": name,
                        "payload": payload})
    unclosed = sum(len(v) for v in open_slices.values())
    if unclosed:
        raise ValueError(f"trace has {unclosed} unclosed slices")
    out.sort(key=lambda e: e["ts_ns"])
    return out


def rank_of(track: str) -> int:
    for part in track.split("/"):
        if part.startswith("rank:"):
            return int(part.split(":", 1)[1])
    raise ValueError(f"track {track!r} names no rank")


def step_statistics(events: list[dict], *, name: str, global_batch_size: int) -> dict[str, Any]:
    """Per-step durations of slices called ``name`` (step from the ``step`` annotation): the slowest
    rank per step, and mean / median / p90 / max over steps with the throughput they imply."""
    per_step: dict[int, float] = {}
    for e in events:
        if e["name"] == name and isinstance(e["payload"].get("step"), int) and e["dur_ns"] > 0:
            s = e["payload"]["step"]
            per_step[s] = max(per_step.get(s, 0.0), e["dur_ns"] / 1e6)
    vals = sorted(per_step.values())
    if not vals:
        return {"count": 0}
    mean = statistics.fmean(vals)
    return {"count": len(vals), "mean_ms": mean, "median_ms": statistics.median(vals),
            "p90_ms": vals[int(0.9 * (len(vals) - 1))], "max_ms": vals[-1],
            "throughput_from_mean_samples_per_sec": global_batch_size / (mean / 1000.0),
            "event_counts": dict(Counter(e["name"] for e in events))}


__all__ = ["PerfettoWriter", "parse_trace", "rank_of", "step_statistics"]
