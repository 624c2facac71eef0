"""Summaries of device traces: kernel time by category, interval unions and overlap.

    python -m flare_b200.utils.trace_summary trace.json          # Chrome trace (torch.profiler export)
    python -m flare_b200.utils.trace_summary launches.csv        # ncu --csv launch list (gpu__time_duration.sum)

Kernels are grouped into categories by name (GEMM, embedding, fused
collective, NCCL, attention, optimizer, elementwise/other).  For a Chrome
trace the summary gives, per category, the kernel count, summed time and the
union of its intervals (time during which at least one such kernel ran, so
concurrent kernels on several streams are not double counted), plus the
overlap of communication with compute.  For an ncu launch list it gives each
kernel's total and share (launches there are serialised, so shares are what
to compare).  Reference behaviour: tools/validation/summarize_jax_profile.py
(interval union, NCCL / GEMM categories) and the phase-overlap analysis in
tools/validation.
"""
from __future__ import annotations

import csv
import json
import re
import sys
from collections import defaultdict
from collections.abc import Iterable

CATEGORIES: tuple[tuple[str, re.Pattern], ...] = (
    ("fused_collective", re.compile(r"gemm_dist|emb_fwd|emb_bwd_pull|adam_dp|tier_|dyn_", re.I)),
    ("nccl", re.compile(r"nccl", re.I)),
    ("attention", re.compile(r"attn|flash|fmha", re.I)),
    ("gemm", re.compile(r"gemm|tcgen05|cutlass|nvjet|sm100_xmma|cublas|matmul", re.I)),
    ("embedding", re.compile(r"emb_|sparse_|unique|scan|segment", re.I)),
    ("optimizer", re.compile(r"adam|adagrad|sgd|optim", re.I)),
)
COMM = ("fused_collective", "nccl")


def categorize(name: str) -> str:
    for cat, pat in CATEGORIES:
        if pat.search(name):
            return cat
    return "other"


def interval_union(intervals: Iterable[tuple[float, float]]) -> float:
    """Total length covered by [start, end) intervals."""
    total, cur_s, cur_e = 0.0, None, None
    for s, e in sorted(intervals):
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                total += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        total += cur_e - cur_s
    return total


def _merge(intervals):
    out = []
    for s, e in sorted(intervals):
        if out and s <= out[-1][1]:
            out[-1][1] = max(out[-1][1], e)
        else:
            out.append([s, e])
    return out


def intersection_length(a: Iterable[tuple[float, float]], b: Iterable[tuple[float, float]]) -> float:
    ma, mb = _merge(a), _merge(b)
    i = j = 0
    tot = 0.0
    while i < len(ma) and j < len(mb):
        s, e = max(ma[i][0], mb[j][0]), min(ma[i][1], mb[j][1])
        if e > s:
            tot += e - s
        if ma[i][1] < mb[j][1]:
            i += 1
        else:
            j += 1
    return tot


def load_chrome_trace(path: str) -> list[dict]:
    """Device kernel events (name, ts, dur in microseconds) of a Chrome trace JSON."""
    with open(path) as f:
        data = json.load(f)
    events = data["traceEvents"] if isinstance(data, dict) else data
    out = []
    for ev in events:
        if ev.get("ph") != "X" or "dur" not in ev:
            continue
        cat = str(ev.get("cat", "")).lower()
        if cat and cat not in ("kernel", "gpu_memcpy", "gpu_memset"):
            continue
        out.append({"name": ev.get("name", ""), "ts": float(ev["ts"]), "dur": float(ev["dur"]),
                    "stream": ev.get("tid")})
    return out


def summarize_events(events: list[dict]) -> dict:
    by: dict[str, list[tuple[float, float]]] = defaultdict(list)
    for ev in events:
        by[categorize(ev["name"])].append((ev["ts"], ev["ts"] + ev["dur"]))
    allv = [iv for v in by.values() for iv in v]
    span = (max(e for _, e in allv) - min(s for s, _ in allv)) if allv else 0.0
    busy = interval_union(allv)
    cats = {}
    for c, iv in sorted(by.items()):
        u = interval_union(iv)
        cats[c] = {"count": len(iv), "sum_us": sum(e - s for s, e in iv), "union_us": u,
                   "share_of_busy": u / busy if busy else 0.0}
    comm = [iv for c in COMM for iv in by.get(c, [])]
    comp = [iv for c, v in by.items() if c not in COMM for iv in v]
    comm_u = interval_union(comm)
    return {"span_us": span, "busy_us": busy, "idle_us": span - busy, "categories": cats,
            "comm_union_us": comm_u,
            "comm_overlapped_us": intersection_length(comm, comp),
            "comm_exposed_us": comm_u - intersection_length(comm, comp)}


def summarize_ncu_csv(path: str, metric: str = "gpu__time_duration.sum") -> dict:
    """Per-kernel totals of an ``ncu --csv`` launch list (one row per launch and metric)."""
    with open(path, newline="") as f:
        lines = [ln for ln in f if ln.startswith('"')]
    rows = list(csv.DictReader(lines))
    tot: dict[str, float] = defaultdict(float)
    cnt: dict[str, int] = defaultdict(int)
    for r in rows:
        if r.get("Metric Name") != metric:
            continue
        unit = r.get("Metric Unit", "")
        v = float(str(r["Metric Value"]).replace(",", ""))
        scale = {"nsecond": 1e-3, "usecond": 1.0, "msecond": 1e3, "second": 1e6}.get(unit, 1e-3)
        name = r.get("Kernel Name", "?")
        tot[name] += v * scale
        cnt[name] += 1
    total = sum(tot.values())
    kernels = sorted(({"kernel": k, "category": categorize(k), "launches": cnt[k], "total_us": t,
                       "share": t / total if total else 0.0} for k, t in tot.items()), key=lambda d: -d["total_us"])
    cats: dict[str, float] = defaultdict(float)
    for k in kernels:
        cats[k["category"]] += k["total_us"]
    return {"total_us": total, "kernels": kernels,
            "categories": {c: {"total_us": t, "share": t / total if total else 0.0} for c, t in cats.items()}}


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        raise SystemExit("usage: python -m flare_b200.utils.trace_summary FILE(.json|.csv)")
    path = argv[0]
    out = summarize_ncu_csv(path) if path.endswith(".csv") else summarize_events(load_chrome_trace(path))
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()


__all__ = ["categorize", "interval_union", "intersection_length", "load_chrome_trace", "summarize_events",
           "summarize_ncu_csv"]
