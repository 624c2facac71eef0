"""How much of a step's side work hides behind its training phase (from a phase timeline).

Input: slices named by phase with an integer ``step`` annotation on tracks
``rank:<r>/<lane>`` (``PerfettoWriter`` output of a ranking graph run, or
any trace with the same naming).  For every selected ``train_core`` slice
and every *relation* -- a phase at a step offset, e.g. the next step's
``prepare_sparse_materialize`` or the previous step's
``scatter_sparse_grads`` -- ``phase_overlap`` reports whether the related
slice exists on that rank, its duration, its overlap with the training
slice and the part of it finished before the training slice ends ("hidden").
``effective_overlap`` summarises the critical relations over all rows and
names what blocks a claim of hidden work (no consistently hidden slices, a
low hidden fraction, more exposed than hidden time).

    python -m flare_b200.validation.overlap trace.pftrace --steps 3,4,5 --out overlap.json

Reference counterparts: tools/validation/analyze_phase_overlap.py and
tools/validation/analyze_effective_overlap.py.
"""
from __future__ import annotations

import argparse
import json
import statistics
from collections import defaultdict
from pathlib import Path
from typing import Any

from .perfetto import parse_trace, rank_of

RELATIONS = {
    "materialize_next": ("prepare_sparse_materialize", 1),
    "bind_next": ("prepare_bind", 1),
    "scatter_prev": ("scatter_sparse_grads", -1),
    "scatter_same": ("scatter_sparse_grads", 0),
    "materialize_same": ("prepare_sparse_materialize", 0),
    "bind_same": ("prepare_bind", 0),
}
CRITICAL = ("materialize_next", "scatter_prev")


def _stat(values: list[float]) -> dict[str, float]:
    if not values:
        return {"count": 0, "total": 0.0}
    v = sorted(values)
    return {"count": len(v), "total": float(sum(v)), "mean": statistics.fmean(v), "median": statistics.median(v),
            "p90": v[int(0.9 * (len(v) - 1))], "min": v[0], "max": v[-1]}


def phase_overlap(events: list[dict], steps: set[int] | None = None, *, train: str = "train_core",
                  relations: dict[str, tuple[str, int]] | None = None) -> dict[str, Any]:
    relations = relations or RELATIONS
    longest: dict[tuple[str, int, int], dict] = {}
    for e in events:
        step = e["payload"].get("step")
        if e["dur_ns"] <= 0 or not isinstance(step, int):
            continue
        key = (e["name"], rank_of(e["track"]), step)
        if key not in longest or e["dur_ns"] > longest[key]["dur_ns"]:
            longest[key] = e
    rows = []
    for (name, rank, step), t in sorted(longest.items(), key=lambda kv: (kv[0][1], kv[0][2])):
        if name != train or (steps is not None and step not in steps):
            continue
        t0, t1 = t["ts_ns"], t["ts_ns"] + t["dur_ns"]
        train_ms = t["dur_ns"] / 1e6
        rel = {}
        for rname, (phase, off) in relations.items():
            c = longest.get((phase, rank, step + off))
            if c is None:
                rel[rname] = {"present": False, "duration_ms": 0.0, "overlap_ms": 0.0, "hidden_ms": 0.0}
                continue
            c0, c1 = c["ts_ns"], c["ts_ns"] + c["dur_ns"]
            dur = c["dur_ns"] / 1e6
            ov = max(0, min(t1, c1) - max(t0, c0)) / 1e6
            hidden = max(0, min(c1, t1) - c0) / 1e6
            rel[rname] = {"present": True, "duration_ms": dur, "overlap_ms": ov, "hidden_ms": hidden,
                          "hidden_fraction_of_candidate": hidden / dur if dur else 0.0,
                          "overlap_fraction_of_train": ov / train_ms if train_ms else 0.0,
                          "starts_before_train_end": c0 < t1, "starts_before_train_start": c0 < t0}
        rows.append({"rank": rank, "step": step, "train_core_ms": train_ms, "overlaps": rel})
    if not rows:
        raise ValueError(f"no {train!r} slices with a step annotation were selected")
    summary = {}
    for rname in relations:
        present = [r["overlaps"][rname] for r in rows if r["overlaps"][rname]["present"]]
        summary[rname] = {"present_count": len(present),
                          "overlap_ms": _stat([p["overlap_ms"] for p in present]),
                          "hidden_fraction_of_candidate": _stat([p["hidden_fraction_of_candidate"] for p in present])}
    return {"rows": rows, "summary": summary}


def effective_overlap(report: dict[str, Any], *, relations=CRITICAL, min_hidden_fraction: float = 0.5,
                      min_positive_count: int = 1) -> dict[str, Any]:
    rows = report["rows"]
    out, blockers = {}, {}
    for rname in relations:
        present = [r["overlaps"][rname] for r in rows if r["overlaps"].get(rname, {}).get("present")]
        dur = [p["duration_ms"] for p in present]
        hid = [p["hidden_ms"] for p in present]
        exposed = [d - h for d, h in zip(dur, hid)]
        total = sum(dur)
        s = {"present_count": len(present), "positive_hidden_count": sum(h > 0 for h in hid),
             "duration_ms": _stat(dur), "hidden_ms": _stat(hid), "exposed_ms": _stat(exposed),
             "total_hidden_fraction": sum(hid) / total if total else 0.0}
        why = []
        if s["positive_hidden_count"] < min_positive_count:
            why.append("no consistently hidden work")
        if s["total_hidden_fraction"] < min_hidden_fraction:
            why.append("low hidden fraction")
        if s["exposed_ms"].get("mean", 0.0) > s["hidden_ms"].get("mean", 0.0):
            why.append("more exposed than hidden")
        out[rname] = s
        if why:
            blockers[rname] = why
    train = [r["train_core_ms"] for r in rows]
    hidden_per_row = [sum(r["overlaps"][n]["hidden_ms"] for n in relations if r["overlaps"].get(n, {}).get("present"))
                      for r in rows]
    return {"relations": out, "train_core_ms": _stat(train),
            "effective_hidden_fraction_of_train": _stat([h / t if t else 0.0 for h, t in zip(hidden_per_row, train)]),
            "blockers": blockers, "overlap_proven": not blockers}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("trace")
    ap.add_argument("--steps", default="", help="comma-separated train_core steps (default: all)")
    ap.add_argument("--out", required=True)
    ap.add_argument("--min-hidden-fraction", type=float, default=0.5)
    args = ap.parse_args(argv)
    steps = {int(s) for s in args.steps.split(",") if s} or None
    rep = phase_overlap(parse_trace(args.trace), steps)
    rep["effective"] = effective_overlap(rep, min_hidden_fraction=args.min_hidden_fraction)
    Path(args.out).write_text(json.dumps(rep, indent=1) + "\n")
    print(json.dumps({"overlap_proven": rep["effective"]["overlap_proven"], "blockers": rep["effective"]["blockers"]}))


if __name__ == "__main__":
    main()


__all__ = ["CRITICAL", "RELATIONS", "effective_overlap", "phase_overlap"]
