"""Host <-> device transfers and zero-copy exchange with other array libraries.

* ``to_host(t)`` starts a device -> host copy into pinned memory on the
  current (or given) stream and returns a ``HostTransfer`` whose ``result()``
  waits on the copy's event only, not on the whole device; pinned buffers are
  reused per (shape, dtype) from a small pool, so a loop that reads back a
  metric every step allocates once.  CPU tensors come back as they are.
* ``from_external(x)`` / ``to_external(t)``: zero-copy views through DLPack
  (any object with ``__dlpack__``, e.g. NumPy or CuPy arrays, or a capsule).

Reference behaviour: src/flare/kernels/conversion.py:30-130 (pinned
non-blocking device -> host copy with an event; DLPack / CUDA array interface
bridging between CuPy, JAX and NumPy).
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

_POOL: dict[tuple, list[torch.Tensor]] = {}
_POOL_LOCK = threading.Lock()
_POOL_PER_KEY = 4


def _pinned(shape: torch.Size, dtype: torch.dtype) -> torch.Tensor:
    key = (tuple(shape), dtype)
    with _POOL_LOCK:
        free = _POOL.get(key)
        if free:
            return free.pop()
    return torch.empty(shape, dtype=dtype, pin_memory=True)


def _release(t: torch.Tensor) -> None:
    key = (tuple(t.shape), t.dtype)
    with _POOL_LOCK:
        free = _POOL.setdefault(key, [])
        if len(free) < _POOL_PER_KEY:
            free.append(t)


@dataclass
class HostTransfer:
    tensor: torch.Tensor
    event: torch.cuda.Event | None = None
    pooled: bool = False

    def ready(self) -> bool:
        return self.event is None or self.event.query()

    def result(self, copy: bool = True) -> torch.Tensor:
        """The host tensor once its copy has landed (a private copy when the buffer is pooled)."""
        if self.event is not None:
            self.event.synchronize()
        if not self.pooled:
            return self.tensor
        out = self.tensor.clone() if copy else self.tensor
        if copy:
            _release(self.tensor)
            self.pooled = False
            self.tensor = out
        return out


def to_host(t: torch.Tensor, stream: torch.cuda.Stream | None = None) -> HostTransfer:
    """Non-blocking device -> pinned host copy ordered on ``stream`` (default: the current stream)."""
    if t.device.type != "cuda":
        return HostTransfer(t.detach())
    s = stream or torch.cuda.current_stream(t.device)
    buf = _pinned(t.shape, t.dtype)
    with torch.cuda.stream(s):
        buf.copy_(t.detach(), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(s)
    return HostTransfer(buf, ev, pooled=True)


def from_external(x) -> torch.Tensor:
    """Zero-copy torch view of a DLPack-capable array (NumPy, CuPy, ...) or a DLPack capsule."""
    return torch.from_dlpack(x)


def to_external(t: torch.Tensor):
    """DLPack capsule of ``t`` (zero copy); e.g. ``numpy.from_dlpack(t)`` also works directly."""
    return torch.utils.dlpack.to_dlpack(t)


__all__ = ["HostTransfer", "from_external", "to_external", "to_host"]
