"""Diagnostics and failure detection (host-side faults only; no GPU fault is caused)."""
import datetime
import json
import os
import time

import pytest
import torch
import torch.distributed as dist

from flare_b200.runtime.diagnostics import JsonlExecutionTracer, fingerprint_state, median_duration_seconds
from flare_b200.runtime.failure import Heartbeat, PeerFailure, PeerWatchdog
from flare_b200.testing.gloo import run_ranks


def test_tracer_and_fingerprint(tmp_path):
    tr = JsonlExecutionTracer(tmp_path, rank=3)
    tr.emit("sparse_update", "apply", grad=torch.tensor([1.0, float("nan"), 2.0]), step=4)
    tr.emit("module_update", "apply", step=4)
    tr.close()
    rec = json.loads((tmp_path / "sparse_update.rank3.jsonl").read_text().splitlines()[0])
    assert rec["grad"]["nan"] == 1 and rec["grad"]["finite"] == 2 and rec["seq"] == 1 and rec["rank"] == 3
    a = fingerprint_state({"w": torch.ones(3), "b": torch.zeros(2)})
    b = fingerprint_state({"b": torch.zeros(2), "w": torch.ones(3)})
    c = fingerprint_state({"w": torch.ones(3), "b": torch.tensor([0.0, 1e-30])})
    assert a["digest"] == b["digest"] != c["digest"] and a["count"] == 2
    assert median_duration_seconds([3, 1, 2]) == 2


def _heartbeat_world(rank, world):
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, interval_s=0.1)
    # margins well above a loaded host's scheduling delays: beats every 0.1 s, silence after 2 s
    dog = PeerWatchdog(store, world, rank, timeout_s=2.0)
    dist.barrier()
    time.sleep(0.3)
    dog.check()  # everyone alive
    dist.barrier()  # both ranks passed the first check before rank 1 goes silent
    if rank == 1:
        hb.stop()  # this rank goes silent (a hang, from the peers' point of view)
        time.sleep(4.0)
        return "silent"
    time.sleep(3.0)
    try:
        dog.check()
    except PeerFailure as e:
        return e.ranks
    return "not detected"


def test_watchdog_detects_silent_rank():
    out = run_ranks(_heartbeat_world, 2)
    assert out[0] == [1] and out[1] == "silent"


def _failing_rank(rank, world):
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, interval_s=0.1)
    dist.barrier()
    if rank == 1:
        try:
            raise ValueError("injected host-side failure")
        except ValueError:
            hb.mark_failed("ValueError")
            return "raised"
    time.sleep(0.5)
    try:
        PeerWatchdog(store, world, rank, timeout_s=30).check()
    except PeerFailure as e:
        return e.ranks
    return "not detected"


def test_watchdog_sees_failure_marker():
    out = run_ranks(_failing_rank, 2)
    assert out == [[1], "raised"]


def _collective_timeout(rank, world):
    # a short process-group timeout ends the survivor's collective with an error
    pg = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=2))
    if rank == 1:
        return "left"
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(1), group=pg)
    except RuntimeError:
        return time.time() - t0
    return "no error"


def test_process_group_timeout_on_missing_peer():
    out = run_ranks(_collective_timeout, 2, timeout=60)
    assert isinstance(out[0], float) and out[0] < 30 and out[1] == "left"


@pytest.mark.gpu
def test_device_wait_times_out_and_context_survives(cuda):
    from flare_b200.runtime.failure import probe_flag_timeout

    t0 = time.time()
    st = probe_flag_timeout(0.2, cuda)
    assert st["code"] == 2 and st["count"] == 1 and time.time() - t0 < 10
    x = torch.ones(1000, device=cuda)
    assert float((x * 2).sum()) == 2000.0  # the context is still usable


def _never_published(rank, world):
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, interval_s=0.1) if rank == 0 else None
    dist.barrier()
    if rank == 1:
        return "never beat"
    t0 = time.monotonic()
    try:
        PeerWatchdog(store, world, rank, timeout_s=30).check()
    except PeerFailure as e:
        return e.ranks, time.monotonic() - t0
    finally:
        hb.stop()
    return "not detected"


def test_watchdog_reports_a_rank_that_never_published_without_waiting():
    out = run_ranks(_never_published, 2)
    ranks, seconds = out[0]
    assert ranks == [1] and seconds < 5.0 and out[1] == "never beat"
