"""Spawn N ranks of a function as local processes with a process group (CPU gloo, or NCCL per GPU).

``spawn_ranks(fn, world, *args)`` starts ``world`` spawned processes, sets
the rendezvous environment (127.0.0.1, a free port), initialises the
process group with a timeout, runs ``fn(rank, world, *args)`` and returns
the ranks' results in rank order.  A rank that raises, exits without
reporting a result (killed, ``os._exit``) or reports nothing before
``timeout`` makes the call raise ``RankFailure`` naming the first failed rank
and its traceback (or exit code), after every process has ended (the
survivors of a lost rank end when their next collective times out).
Results travel as ``torch.save`` bytes, so tensors do not depend on the
sender process staying alive.
"""
from __future__ import annotations

import datetime
import io
import os
import queue
import socket
import time
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class RankFailure(RuntimeError):
    def __init__(self, rank: int, detail: str, failed: dict[int, str]):
        super().__init__(f"rank {rank} failed:\n{detail}")
        self.rank, self.detail, self.failed = rank, detail, failed


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, backend, pg_timeout_s, fn, args, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout_s))
        out = fn(rank, world, *args)
        buf = io.BytesIO()
        torch.save(out, buf)
        queue.put((rank, "ok", buf.getvalue()))
    except BaseException:  # noqa: BLE001 - report any failure to the parent
        queue.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001 - a broken group after a peer's loss
                pass


def spawn_ranks(fn, world: int, *args, backend: str = "gloo", timeout: float = 120.0,
                pg_timeout_s: float = 60.0) -> list:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, backend, pg_timeout_s, fn, args, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results, failed = {}, {}
    pending = set(range(world))

    def take(item):
        rank, status, out = item
        pending.discard(rank)
        if status == "ok":
            results[rank] = torch.load(io.BytesIO(out), weights_only=False)
        else:
            failed[rank] = out

    deadline = time.monotonic() + timeout
    try:
        while pending:
            left = deadline - time.monotonic()
            if left <= 0:
                for r in sorted(pending):
                    failed[r] = f"no result within {timeout:.0f} s"
                break
            try:
                take(q.get(timeout=min(1.0, left)))
                continue
            except queue.Empty:
                pass
            dead = [r for r in sorted(pending) if not procs[r].is_alive()]
            if not dead:
                continue
            # a result is in the pipe before its process exits: drain, then whoever is still missing
            # exited without reporting (killed, os._exit, a crash below Python)
            while True:
                try:
                    take(q.get_nowait())
                except queue.Empty:
                    break
            for r in dead:
                if r in pending:
                    pending.discard(r)
                    failed[r] = f"exited with code {procs[r].exitcode} without reporting a result"
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    if failed:
        first = min(failed)
        raise RankFailure(first, failed[first], failed)
    return [results[r] for r in range(world)]


__all__ = ["RankFailure", "free_port", "spawn_ranks"]
