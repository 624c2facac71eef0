"""Sparse precision contracts ("numerical rescue").

Same contract as the reference (src/flare/runtime/sparse_precision.py:8-17):
table values are stored as float16 or float32; gradients travel between ranks
as bfloat16 or float32; the native gradient accumulation and the optimizer
state are always float32.  In this framework the bf16 -> fp32 promotion and the
fp32 accumulation happen inside the fused backward kernel.
"""
from __future__ import annotations

import torch

SPARSE_FLOAT16_DTYPE = "float16"
SPARSE_BFLOAT16_DTYPE = "bfloat16"
SPARSE_FLOAT32_DTYPE = "float32"
SPARSE_VALUE_DTYPES = frozenset({SPARSE_FLOAT16_DTYPE, SPARSE_FLOAT32_DTYPE, SPARSE_BFLOAT16_DTYPE})
SPARSE_GRADIENT_TRANSPORT_DTYPES = frozenset({SPARSE_BFLOAT16_DTYPE, SPARSE_FLOAT32_DTYPE})
SPARSE_GRADIENT_DTYPES = frozenset({SPARSE_FLOAT32_DTYPE})
SPARSE_OPTIMIZER_DTYPES = frozenset({SPARSE_FLOAT32_DTYPE})
SPARSE_NATIVE_GRADIENT_DTYPE = SPARSE_FLOAT32_DTYPE
SPARSE_KEY_DTYPES = frozenset({"int32", "int64"})

TORCH_DTYPES = {
    SPARSE_FLOAT16_DTYPE: torch.float16,
    SPARSE_BFLOAT16_DTYPE: torch.bfloat16,
    SPARSE_FLOAT32_DTYPE: torch.float32,
    "int32": torch.int32,
    "int64": torch.int64,
}


def _require(value, allowed, field):
    if not isinstance(value, str) or value not in allowed:
        raise ValueError(f"{field} must be one of {sorted(allowed)!r}, got {value!r}")
    return value


def require_sparse_value_dtype(value):
    return _require(value, SPARSE_VALUE_DTYPES, "sparse embedding value_dtype")


def require_sparse_gradient_dtype(value):
    return _require(value, SPARSE_GRADIENT_DTYPES, "sparse embedding gradient_dtype")


def require_sparse_gradient_transport_dtype(value):
    return _require(value, SPARSE_GRADIENT_TRANSPORT_DTYPES, "sparse embedding gradient_transport_dtype")


def require_sparse_optimizer_dtype(value):
    return _require(value, SPARSE_OPTIMIZER_DTYPES, "sparse embedding optimizer_dtype")


def require_key_dtype(value):
    return _require(value, SPARSE_KEY_DTYPES, "sparse embedding key_dtype")


def require_sparse_key_dtype(values: torch.Tensor, key_dtype: str, *, boundary: str) -> torch.Tensor:
    expected = TORCH_DTYPES[require_key_dtype(key_dtype)]
    if values.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"sparse key dtype at {boundary} must be int32 or int64, got {values.dtype}")
    if values.dtype != expected:
        raise TypeError(f"sparse key dtype mismatch at {boundary}: expected={expected}, got={values.dtype}")
    return values


def require_sparse_tensor_dtype(values: torch.Tensor, dtype: str, *, boundary: str) -> torch.Tensor:
    if dtype not in SPARSE_VALUE_DTYPES | SPARSE_GRADIENT_TRANSPORT_DTYPES:
        raise ValueError(f"sparse precision check requires float16, bfloat16 or float32, got {dtype!r}")
    if values.dtype != TORCH_DTYPES[dtype]:
        raise TypeError(
            f"sparse precision check dtype mismatch at {boundary}: expected={dtype} actual={values.dtype}")
    return values


def require_finite_sparse_values(values: torch.Tensor, dtype: str, *, boundary: str) -> torch.Tensor:
    """Explicit (opt-in, host-synchronising) finite check."""
    require_sparse_tensor_dtype(values, dtype, boundary=boundary)
    if not bool(torch.isfinite(values).all()):
        raise FloatingPointError(f"non-finite sparse values at {boundary}")
    return values


def prepare_sparse_native_gradient(values: torch.Tensor, *, transport_dtype: str, native_dtype: str,
                                   validate_values: bool = False) -> torch.Tensor:
    require_sparse_gradient_transport_dtype(transport_dtype)
    require_sparse_gradient_dtype(native_dtype)
    if values.dtype != TORCH_DTYPES[transport_dtype]:
        raise TypeError(
            f"sparse gradient transport dtype mismatch: expected={transport_dtype} actual={values.dtype}")
    if not isinstance(validate_values, bool):
        raise TypeError("validate_values must be bool")
    out = values.to(TORCH_DTYPES[native_dtype])
    if validate_values:
        require_finite_sparse_values(out, native_dtype, boundary="sparse_native_gradient")
    return out


__all__ = [name for name in dir() if name.startswith(("SPARSE_", "require_", "prepare_"))] + ["TORCH_DTYPES"]
