"""Run a function on N CPU ranks over gloo (multi-process tests without a GPU)."""
from __future__ import annotations

from ..runtime.launch import RankFailure, free_port, spawn_ranks


def run_ranks(fn, world: int, *args, timeout: float = 120.0):
    """Returns [result of rank 0, ..., rank world-1]; raises if any rank failed."""
    try:
        return spawn_ranks(fn, world, *args, backend="gloo", timeout=timeout)
    except RankFailure as e:
        raise RuntimeError(str(e)) from e


__all__ = ["exit_silently_worker", "free_port", "run_ranks"]


def exit_silently_worker(rank: int, world: int, exit_rank: int = 1, code: int = 3):
    """Rank ``exit_rank`` leaves with ``os._exit(code)`` (no exception, no result) while a world
    larger than one; the others return their rank.  Host-side failure for the launcher tests."""
    import os

    if world > 1 and rank == exit_rank:
        os._exit(code)
    return rank
