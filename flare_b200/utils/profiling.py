"""Per-rank device traces of a few steady-state steps (torch.profiler -> Chrome trace -> summary).

    from flare_b200.utils.profiling import profile_steps
    report = profile_steps(lambda: trainer.train_step(batch), steps=3, warmup=5, out_dir="traces", rank=rank)

Runs ``warmup`` untraced steps (allocator, module load, CUDA-graph capture),
then traces ``steps`` steps with CPU and CUDA activities, each inside a
``flare_step_<i>`` range, writes ``<out_dir>/rank<r>.json`` (Chrome trace
format, readable by Perfetto) and returns the kernel summary of
``flare_b200.utils.trace_summary`` (time per category, interval unions,
communication overlap).  One file per rank, as the reference's profiling
workflow writes one directory per rank after a warm-up and a fence
(docs/jax_profiling.md:7-40; profiler config with skip-initial-steps and
steady-state-only, recipes/recsys/ranking/profiler.py:16-60).  Numbers taken
under a profiler are for attribution, not for reporting throughput.
"""
from __future__ import annotations

from collections.abc import Callable
from pathlib import Path

import torch

from .trace_summary import load_chrome_trace, summarize_events


def profile_steps(step: Callable[[], object], *, steps: int = 3, warmup: int = 3, out_dir: str | Path = "traces",
                  rank: int = 0) -> dict:
    from torch.profiler import ProfilerActivity, profile, record_function

    for _ in range(warmup):
        step()
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.synchronize()
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if cuda else [])
    with profile(activities=acts, acc_events=True) as prof:
        for i in range(steps):
            with record_function(f"flare_step_{i}"):
                step()
        if cuda:
            torch.cuda.synchronize()
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    path = out / f"rank{rank}.json"
    prof.export_chrome_trace(str(path))
    summary = summarize_events(load_chrome_trace(str(path)))
    summary["trace"] = str(path)
    summary["steps"] = steps
    return summary


__all__ = ["profile_steps"]
