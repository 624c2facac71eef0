"""Replay a semantic execution trace and check it (the sparse-training audit).

    python -m flare_b200.utils.trace_audit TRACE_DIR        # exit 1 when a check fails

Reads every ``<stage>.rank<r>.jsonl`` file that ``JsonlExecutionTracer``
wrote (``DLRM.traced_step`` emits the stages below) and checks, per rank:

* sequence numbers are unique and increasing across all stage files;
* every traced step has every stage, in pipeline order;
* no tensor summary reports a NaN or an Inf;
* the sparse update's counters are consistent (occurrences >= unique rows
  >= heavy rows >= 0) and the lookup saw the ids the input stage staged;
* the optimizer step counters advance by one per traced step.

Reference behaviour: tools/validation/audit_sparse_training.py:12-20, which
replays the recsys execution trace (recipes/recsys/ranking/metrics/
execution_trace.py:75-380) to check the numerics of a run.
"""
from __future__ import annotations

import json
import re
import sys
from collections import defaultdict
from pathlib import Path

STAGES = ("input_unique", "sparse_lookup", "module_gather", "module_gradient", "sparse_update", "module_update",
          "sparse_commit")


def load_trace(directory: str | Path) -> dict[int, list[dict]]:
    """rank -> events sorted by sequence number."""
    by_rank: dict[int, list[dict]] = defaultdict(list)
    for f in sorted(Path(directory).glob("*.rank*.jsonl")):
        m = re.match(r"(.+)\.rank(\d+)\.jsonl$", f.name)
        if not m:
            continue
        with f.open() as fh:
            for line in fh:
                line = line.strip()
                if line:
                    by_rank[int(m.group(2))].append(json.loads(line))
    return {r: sorted(ev, key=lambda e: e["seq"]) for r, ev in by_rank.items()}


def _summaries(obj, path=""):
    """(path, summary) for every tensor summary nested in an event."""
    if isinstance(obj, dict):
        if "dtype" in obj and "shape" in obj:
            yield path, obj
            return
        for k, v in obj.items():
            yield from _summaries(v, f"{path}.{k}" if path else k)
    elif isinstance(obj, list):
        for i, v in enumerate(obj):
            yield from _summaries(v, f"{path}[{i}]")


def audit_events(events: list[dict]) -> list[str]:
    problems = []
    seqs = [e["seq"] for e in events]
    if len(set(seqs)) != len(seqs):
        problems.append("duplicate sequence numbers")
    steps: dict[int, list[dict]] = defaultdict(list)
    for e in events:
        if "step" in e:
            steps[int(e["step"])].append(e)
        for path, s in _summaries(e):
            if s.get("nan", 0) or s.get("inf", 0):
                problems.append(f"step {e.get('step')} {e['stage']}.{path}: {s.get('nan', 0)} NaN, {s.get('inf', 0)} Inf")
    last_commit = None
    for st in sorted(steps):
        evs = steps[st]
        order = [e["stage"] for e in evs]
        missing = [x for x in STAGES if x not in order]
        if missing:
            problems.append(f"step {st}: missing stages {missing}")
            continue
        if [x for x in order if x in STAGES] != list(STAGES):
            problems.append(f"step {st}: stages out of order {order}")
        ev = {e["stage"]: e for e in evs}
        up = ev["sparse_update"]
        u, occ, heavy = up.get("unique_rows", 0), up.get("occurrences", 0), up.get("heavy_rows", 0)
        if not occ >= u >= heavy >= 0:
            problems.append(f"step {st}: inconsistent sparse update counters {u=} {occ=} {heavy=}")
        if occ > ev["input_unique"].get("ids", occ):
            problems.append(f"step {st}: the update saw {occ} occurrences of {ev['input_unique']['ids']} staged ids")
        c = ev["sparse_commit"]
        cur = (c.get("sparse_optimizer_step"), c.get("dense_optimizer_step"))
        if last_commit is not None and (cur[0] != last_commit[0] + 1 or cur[1] != last_commit[1] + 1):
            problems.append(f"step {st}: optimizer steps {cur} do not follow {last_commit}")
        last_commit = cur
    return problems


def audit_trace(directory: str | Path) -> dict:
    trace = load_trace(directory)
    per_rank = {r: audit_events(ev) for r, ev in trace.items()}
    steps = {r: len({e["step"] for e in ev if "step" in e}) for r, ev in trace.items()}
    return {"ok": bool(trace) and not any(per_rank.values()), "ranks": sorted(trace), "steps": steps,
            "problems": {r: p for r, p in per_rank.items() if p}}


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        raise SystemExit("usage: python -m flare_b200.utils.trace_audit TRACE_DIR")
    rep = audit_trace(argv[0])
    print(json.dumps(rep, indent=1))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())


__all__ = ["STAGES", "audit_events", "audit_trace", "load_trace"]
