"""Precision policy (closed set fp32 / bf16 / fp16).

Same contract as the reference's PrecisionPolicy
(src/flare/jax/training/precision.py:15-99): mixed precision computes in a
low-precision view, transports gradients in bf16 (fp32 exponent range), and
keeps master weights, optimizer state and gradient accumulation in fp32;
dynamic sparse tables store fp16 values under mixed precision and fp32
otherwise, with fp32 sparse gradients and optimizer state.  In this framework
the bf16 compute view is the flat ``compute`` copy, the fp32 master is the
flat ``master`` buffer, and the sparse fp32 accumulation happens inside the
fused backward kernel.
"""
from __future__ import annotations

from enum import Enum

import torch

from ..sparse.precision import SPARSE_FLOAT16_DTYPE, SPARSE_FLOAT32_DTYPE, SPARSE_NATIVE_GRADIENT_DTYPE


class PrecisionPolicy(str, Enum):
    FP32 = "fp32"
    BF16 = "bf16"
    FP16 = "fp16"

    @classmethod
    def fp32(cls) -> "PrecisionPolicy":
        return cls.FP32

    @classmethod
    def bf16(cls) -> "PrecisionPolicy":
        return cls.BF16

    @classmethod
    def fp16(cls) -> "PrecisionPolicy":
        return cls.FP16

    @property
    def compute_dtype(self) -> torch.dtype:
        return {PrecisionPolicy.FP32: torch.float32, PrecisionPolicy.BF16: torch.bfloat16,
                PrecisionPolicy.FP16: torch.float16}[self]

    @property
    def parameter_dtype(self) -> torch.dtype:
        return torch.float32

    @property
    def optimizer_dtype(self) -> torch.dtype:
        return torch.float32

    @property
    def gradient_transport_dtype(self) -> torch.dtype:
        return torch.float32 if self is PrecisionPolicy.FP32 else torch.bfloat16

    @property
    def sparse_storage_dtype_name(self) -> str:
        return SPARSE_FLOAT32_DTYPE if self is PrecisionPolicy.FP32 else SPARSE_FLOAT16_DTYPE

    @property
    def sparse_optimizer_dtype_name(self) -> str:
        return SPARSE_FLOAT32_DTYPE

    @property
    def sparse_gradient_dtype_name(self) -> str:
        return SPARSE_NATIVE_GRADIENT_DTYPE

    @property
    def sparse_gradient_transport_dtype_name(self) -> str:
        return "float32" if self is PrecisionPolicy.FP32 else "bfloat16"


# ------------------------------------------------------------ fp32 islands and constants
class Fp32Island(torch.nn.Module):
    """Runs the wrapped module in fp32 whatever the surrounding autocast: floating inputs are cast
    to fp32 and autocast is off inside (the compute view of the reference's ``Fp32Param``, whose
    parameters keep their fp32 view under mixed precision; src/flare/jax/roles.py:11)."""

    def __init__(self, inner: torch.nn.Module):
        super().__init__()
        self.inner = inner

    def forward(self, *args, **kwargs):
        cast = lambda x: x.float() if torch.is_tensor(x) and x.is_floating_point() else x  # noqa: E731
        dev = next((a.device.type for a in args if torch.is_tensor(a)), "cpu")
        with torch.autocast(device_type=dev, enabled=False):
            return self.inner(*[cast(a) for a in args], **{k: cast(v) for k, v in kwargs.items()})


def register_constant(module: torch.nn.Module, name: str, value: torch.Tensor) -> None:
    """An immutable, non-trainable tensor carried as module state (the reference's
    ``ConstantBuffer``, src/flare/jax/roles.py:15): a persistent buffer, checkpointed, never averaged
    across ranks, and checked for mutation when the engine runs with ``validate_constants``."""
    module.register_buffer(name, value, persistent=True)
    names = module.__dict__.setdefault("_flare_constants", set())
    names.add(name)


def constant_buffers(model: torch.nn.Module) -> dict[str, torch.Tensor]:
    """Every registered constant of ``model`` by its dotted buffer name."""
    out = {}
    for prefix, m in model.named_modules():
        for n in m.__dict__.get("_flare_constants", ()):
            out[f"{prefix}.{n}" if prefix else n] = getattr(m, n)
    return out


__all__ = ["Fp32Island", "PrecisionPolicy", "constant_buffers", "register_constant"]
