"""HTTP session with retries (5xx, connect/read errors, exponential backoff) and TCP keep-alive.

One session per process: a session created before a fork would share its
pooled sockets with the children, so ``get_process_http_session`` rebuilds
it when the process id changes.  Reference behaviour: src/flare/io/http.py:
20-110.
"""
from __future__ import annotations

import os
import socket

import requests
from requests.adapters import HTTPAdapter
from urllib3.util.retry import Retry


def keepalive_socket_options() -> list[tuple[int, int, int]]:
    opts = [(socket.SOL_SOCKET, socket.SO_KEEPALIVE, 1)]
    for name, val in (("TCP_KEEPIDLE", 60), ("TCP_KEEPINTVL", 10), ("TCP_KEEPCNT", 6)):
        if hasattr(socket, name):
            opts.append((socket.IPPROTO_TCP, getattr(socket, name), val))
    return opts


class KeepAliveAdapter(HTTPAdapter):
    def init_poolmanager(self, *args, **kwargs):
        kwargs["socket_options"] = keepalive_socket_options()
        return super().init_poolmanager(*args, **kwargs)

    def proxy_manager_for(self, *args, **kwargs):
        kwargs["socket_options"] = keepalive_socket_options()
        return super().proxy_manager_for(*args, **kwargs)


def create_retry_session(max_retries: int = 5, backoff_factor: float = 1.0) -> requests.Session:
    s = requests.Session()
    retry = Retry(total=max_retries, connect=max_retries, read=max_retries, backoff_factor=backoff_factor,
                  status_forcelist=(500, 502, 503, 504))
    adapter = KeepAliveAdapter(max_retries=retry, pool_connections=32, pool_maxsize=32)
    s.mount("http://", adapter)
    s.mount("https://", adapter)
    return s


_SESSION: requests.Session | None = None
_PID: int | None = None


def get_process_http_session() -> requests.Session:
    global _SESSION, _PID
    if _SESSION is None or _PID != os.getpid():
        _SESSION, _PID = create_retry_session(), os.getpid()
    return _SESSION


__all__ = ["KeepAliveAdapter", "create_retry_session", "get_process_http_session", "keepalive_socket_options"]
