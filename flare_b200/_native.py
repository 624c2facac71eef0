"""Loader for the in-tree native extension ``flare_b200._C`` (sm_100a).

On a machine with a CUDA device the extension is mandatory: every CUDA op in
this package calls it and raises if it is missing, so GPU runs never fall back
silently to PyTorch code. Without a CUDA device the CPU reference paths of the
ops are used instead (those are the numerics oracles and the CPU/gloo
configuration).
"""
from __future__ import annotations

import importlib

import torch

_C = None
_IMPORT_ERROR: Exception | None = None

try:  # pragma: no cover - exercised on GPU boxes
    _C = importlib.import_module("flare_b200._C")
except Exception as exc:  # noqa: BLE001 - report the original failure later
    _IMPORT_ERROR = exc


def native():
    """Return the native module or raise a descriptive error."""
    if _C is None:
        raise RuntimeError(
            "flare_b200 native extension is not built or failed to load "
            f"({_IMPORT_ERROR!r}); run `python setup.py build_ext --inplace`"
        )
    return _C


def available() -> bool:
    return _C is not None


def on_cuda(*tensors: torch.Tensor) -> bool:
    """True when the op must take the CUDA path (and therefore needs _C)."""
    cuda = [t.is_cuda for t in tensors if isinstance(t, torch.Tensor)]
    if any(cuda) and not all(cuda):
        raise ValueError("all tensors of one op must be on the same device type")
    return bool(cuda) and all(cuda)


DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {dt}") from exc


class DeviceStatus:
    """int32[4] device status word written by kernels with bounded waits.

    [0] first error code, [1] detail, [2] error count. ``check()`` reads it back
    (a device->host sync) and raises on any recorded error.
    """

    CODES = {
        1: "mbarrier wait timed out",
        2: "peer signal wait timed out",
        3: "index out of range",
        4: "staging capacity overflow",
        5: "bad argument",
    }

    def __init__(self, device: torch.device):
        self.buf = torch.zeros(4, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def check(self, what: str = "kernel") -> None:
        vals = self.buf.tolist()
        if vals[0] != 0:
            msg = self.CODES.get(vals[0], f"error code {vals[0]}")
            self.buf.zero_()
            raise RuntimeError(f"{what}: {msg} (detail={vals[1]}, count={vals[2]})")

    def reset(self) -> None:
        self.buf.zero_()


_STATUS: dict[int, DeviceStatus] = {}


def default_status(device: torch.device) -> DeviceStatus:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STATUS:
        _STATUS[idx] = DeviceStatus(torch.device("cuda", idx))
    return _STATUS[idx]


DEFAULT_TIMEOUT_NS = 2_000_000_000        # waits inside one CTA (mbarrier phases)
import os as _os

# waits on another GPU's signal (absorbs host-side skew); FLARE_PEER_TIMEOUT_S overrides
PEER_TIMEOUT_NS = int(float(_os.environ.get("FLARE_PEER_TIMEOUT_S", "30")) * 1e9)
