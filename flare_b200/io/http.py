"""HTTP access for config / auth / artifact endpoints: pooled, kept alive, retried.

Connections are described by a :class:`HttpSettings` value (pool size, TCP
keep-alive timing, retry budget and which statuses count as transient).  A
session built from it keeps idle pooled sockets alive with TCP keep-alive
probes, and retries connection errors, read errors and the transient server
statuses with exponential back-off.

``process_session(settings)`` hands out one session per (process, settings):
pooled sockets must not be shared across ``fork``, so a child process gets
its own.  Reference behaviour: src/flare/io/http.py:20-110 (a retrying,
keep-alive session cached per process).
"""
from __future__ import annotations

import os
import socket
import threading
from dataclasses import dataclass

import requests
from requests.adapters import HTTPAdapter
from urllib3.util.retry import Retry


@dataclass(frozen=True)
class HttpSettings:
    pool_size: int = 32
    keepalive_idle_s: int = 45      # idle time before the first probe
    keepalive_interval_s: int = 15  # between probes
    keepalive_probes: int = 4       # unanswered probes before the socket is dropped
    retries: int = 5
    backoff_s: float = 1.0          # first back-off; doubles per attempt
    transient_statuses: tuple[int, ...] = (500, 502, 503, 504)

    def socket_options(self) -> list[tuple[int, int, int]]:
        """setsockopt triples: keep-alive on, with the timings this platform lets us set."""
        wanted = {"TCP_KEEPIDLE": self.keepalive_idle_s, "TCP_KEEPINTVL": self.keepalive_interval_s,
                  "TCP_KEEPCNT": self.keepalive_probes}
        opts = [(socket.SOL_SOCKET, socket.SO_KEEPALIVE, 1)]
        opts += [(socket.IPPROTO_TCP, getattr(socket, k), v) for k, v in wanted.items() if hasattr(socket, k)]
        return opts

    def retry(self) -> Retry:
        n = self.retries
        return Retry(total=n, connect=n, read=n, backoff_factor=self.backoff_s,
                     status_forcelist=self.transient_statuses, allowed_methods=None)


class _KeepAlivePool(HTTPAdapter):
    """An adapter whose direct and proxied connection pools open sockets with keep-alive options."""

    def __init__(self, settings: HttpSettings):
        self._sockopts = settings.socket_options()
        super().__init__(max_retries=settings.retry(), pool_connections=settings.pool_size,
                         pool_maxsize=settings.pool_size)

    def init_poolmanager(self, *args, **kwargs):
        kwargs.setdefault("socket_options", self._sockopts)
        return super().init_poolmanager(*args, **kwargs)

    def proxy_manager_for(self, *args, **kwargs):
        kwargs.setdefault("socket_options", self._sockopts)
        return super().proxy_manager_for(*args, **kwargs)


def make_session(settings: HttpSettings | None = None) -> requests.Session:
    """A new session with keep-alive pooling and retries on both schemes."""
    settings = settings or HttpSettings()
    session = requests.Session()
    adapter = _KeepAlivePool(settings)
    for scheme in ("http://", "https://"):
        session.mount(scheme, adapter)
    return session


_sessions: dict[tuple[int, HttpSettings], requests.Session] = {}
_sessions_lock = threading.Lock()


def process_session(settings: HttpSettings | None = None) -> requests.Session:
    """The session of this process for ``settings`` (a forked child builds its own)."""
    key = (os.getpid(), settings or HttpSettings())
    with _sessions_lock:
        s = _sessions.get(key)
        if s is None:
            for stale in [k for k in _sessions if k[0] != key[0]]:
                del _sessions[stale]  # inherited from the parent: its sockets are not ours
            s = _sessions[key] = make_session(key[1])
        return s


def create_retry_session(max_retries: int = 5, backoff_factor: float = 1.0) -> requests.Session:
    """A session with the given retry budget and first back-off (other settings: defaults)."""
    return make_session(HttpSettings(retries=max_retries, backoff_s=backoff_factor))


def get_process_http_session() -> requests.Session:
    """The default-settings session of this process."""
    return process_session()


__all__ = ["HttpSettings", "create_retry_session", "get_process_http_session", "make_session", "process_session"]
