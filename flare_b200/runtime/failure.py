"""Failure detection: host heartbeats, a peer watchdog, device status checks.

* ``Heartbeat`` publishes ``(timestamp, step)`` for this rank into the
  torch.distributed key-value store from a background thread.
* ``PeerWatchdog.check()`` reads every peer's heartbeat and raises
  ``PeerFailure`` naming the ranks that are stale beyond ``timeout_s``, that
  never published, or that published a failure marker (without blocking on a
  missing key); training loops call it between steps, before
  launching kernels that wait on peers, so a dead peer is found on the host
  instead of by a device wait running out.
* Device waits are bounded (see csrc/common.cuh): a wait that runs out records
  an error code in a status word and the kernel returns; ``DeviceStatus.check``
  raises on the host.  ``probe_flag_timeout`` exercises that path with a flag
  nothing sets.

Reference mechanisms: Fluxway heartbeats (recipes/recsys/ranking/benchmark/
runner.py:220-222) and per-operator process-group timeouts.
"""
from __future__ import annotations

import threading
import time

import torch
import torch.distributed as dist


class PeerFailure(RuntimeError):
    def __init__(self, ranks: list[int], reason: str):
        super().__init__(f"peer ranks {ranks} failed: {reason}")
        self.ranks = ranks


def _key(rank: int) -> str:
    return f"flare_b200/heartbeat/{rank}"


class Heartbeat:
    def __init__(self, store: dist.Store, rank: int, interval_s: float = 1.0):
        self.store, self.rank, self.interval = store, rank, interval_s
        self.step = 0
        self._stop = threading.Event()
        self._publish()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _publish(self, status: str = "ok") -> None:
        self.store.set(_key(self.rank), f"{time.time()}|{self.step}|{status}")

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._publish()
            except Exception:  # noqa: BLE001 - store gone: nothing to report to
                return

    def set_step(self, step: int) -> None:
        self.step = int(step)

    def mark_failed(self, reason: str = "error") -> None:
        self._stop.set()
        try:
            self._publish(f"failed:{reason}")
        except Exception:  # noqa: BLE001
            pass

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)


class PeerWatchdog:
    def __init__(self, store: dist.Store, world_size: int, rank: int, timeout_s: float = 10.0):
        self.store, self.world, self.rank, self.timeout = store, world_size, rank, timeout_s

    def check(self) -> None:
        now = time.time()
        stale, failed = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            # a store's get() waits for a missing key up to the store's own timeout (minutes for a
            # TCPStore): ask whether it exists first, so a rank that never published is reported now
            try:
                raw = self.store.get(_key(r)).decode() if self.store.check([_key(r)]) else None
            except Exception:  # noqa: BLE001 - store unreachable or key gone
                raw = None
            if raw is None:
                stale.append(r)
                continue
            ts, _, status = raw.split("|", 2)
            if status.startswith("failed"):
                failed.append(r)
            elif now - float(ts) > self.timeout:
                stale.append(r)
        if failed:
            raise PeerFailure(failed, "peer reported a failure")
        if stale:
            raise PeerFailure(stale, f"no heartbeat for more than {self.timeout}s")


def probe_flag_timeout(timeout_s: float = 0.2, device: torch.device | None = None) -> dict:
    """Launch a device wait on a flag nothing sets; return the status it recorded."""
    from .._native import DeviceStatus, native

    dev = device or torch.device("cuda", torch.cuda.current_device())
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    st = DeviceStatus(dev)
    native().wait_flag_probe(flag.data_ptr(), 1, int(timeout_s * 1e9), st.ptr)
    torch.cuda.synchronize(dev)
    code, detail, count, _ = st.buf.tolist()
    return {"code": code, "detail": detail, "count": count}


__all__ = ["Heartbeat", "PeerFailure", "PeerWatchdog", "probe_flag_timeout"]
