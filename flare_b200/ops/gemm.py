"""bf16 GEMM on tcgen05 tensor cores with fused epilogues.

``gemm(a, b)`` computes ``C[M,N] = alpha * A[M,K] @ B[N,K]^T`` where ``A`` is
``a`` (row-major ``[M,K]``) or ``a.T`` when ``a_t`` (``a`` stored ``[K,M]``), and
likewise for ``B``.  Transposed operands go to the tensor core through the
descriptor's MN-major mode; nothing is copied.

Epilogue options: ``bias`` (bf16 ``[N]``), ``relu``, ``mask`` (bf16 ``[M,N]``:
result is zeroed where ``mask <= 0``, i.e. ReLU backward), ``colsum`` (fp32
``[N]`` accumulates the column sums of the result: bias gradient), and fp32
output with ``accumulate`` (gradient accumulation).

``pair=True`` runs tiles of at least 256 x 128 on CTA pairs (``cta_group::2``:
two SMs share one 256-row MMA, each staging half of the operands), ``False``
never, ``None`` as the ``FLARE_GEMM_PAIR`` environment variable says (``1``).

CUDA tensors run the native kernel; CPU tensors run the fp32 reference below
(also the oracle in the numerics tests).  The reference computes its dense
layers through XLA/cuBLAS (src/flare/jax/layers/base.py:27 MLP).
"""
from __future__ import annotations

import torch

from .._native import DEFAULT_TIMEOUT_NS, default_status, native, on_cuda

F32, BF16 = 0, 1


def _logical(t: torch.Tensor, transposed: bool) -> tuple[int, int, int]:
    """Return (rows, K, ld) of the logical [rows, K] operand."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("GEMM operands must be 2-D with unit inner stride")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"GEMM operands must be bfloat16, got {t.dtype}")
    if transposed:
        return t.shape[1], t.shape[0], t.stride(0)
    return t.shape[0], t.shape[1], t.stride(0)


def gemm_reference(a, b, *, a_t=False, b_t=False, bias=None, relu=False, alpha=1.0, mask=None):
    A = (a.t() if a_t else a).float()
    B = (b.t() if b_t else b).float()
    c = alpha * (A @ B.t())
    if bias is not None:
        c = c + bias.float()
    if relu:
        c = torch.relu(c)
    if mask is not None:
        c = torch.where(mask.float() > 0, c, torch.zeros_like(c))
    return c


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_t: bool = False,
    b_t: bool = False,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    relu: bool = False,
    alpha: float = 1.0,
    mask: torch.Tensor | None = None,
    colsum: torch.Tensor | None = None,
    accumulate: bool = False,
    bn: int = 0,
    pair: bool | None = None,
) -> torch.Tensor:
    M, K, lda = _logical(a, a_t)
    N, Kb, ldb = _logical(b, b_t)
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    if out is None:
        if accumulate:
            raise ValueError("accumulate requires an output tensor")
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if out.dtype not in (torch.float32, torch.bfloat16) or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("bad GEMM output tensor")
    if accumulate and out.dtype != torch.float32:
        raise ValueError("accumulate requires an fp32 output")
    if mask is not None and (mask.shape != (M, N) or mask.dtype != torch.bfloat16 or mask.stride(1) != 1):
        raise ValueError("mask must be bf16 [M, N]")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != N):
        raise ValueError("bias must be bf16 [N]")
    if colsum is not None and (colsum.dtype != torch.float32 or colsum.numel() != N):
        raise ValueError("colsum must be fp32 [N]")

    if not on_cuda(a, b, out):
        c = gemm_reference(a, b, a_t=a_t, b_t=b_t, bias=bias, relu=relu, alpha=alpha, mask=mask)
        if colsum is not None:
            colsum += c.sum(0)
        if accumulate:
            out += c
        else:
            out.copy_(c.to(out.dtype))
        return out

    C = native()
    st = default_status(a.device)
    C.gemm(
        A=a.data_ptr(), lda=lda, a_mn=a_t,
        B=b.data_ptr(), ldb=ldb, b_mn=b_t,
        M=M, N=N, K=K,
        C=out.data_ptr(), ldc=out.stride(0), c_dtype=F32 if out.dtype == torch.float32 else BF16,
        accumulate=accumulate,
        bias=bias.data_ptr() if bias is not None else 0,
        act=1 if relu else 0, alpha=float(alpha),
        mask=mask.data_ptr() if mask is not None else 0, ldm=mask.stride(0) if mask is not None else 0,
        colsum=colsum.data_ptr() if colsum is not None else 0,
        status=st.ptr, timeout_ns=DEFAULT_TIMEOUT_NS, bn=bn, pair=-1 if pair is None else int(bool(pair)),
    )
    return out


__all__ = ["gemm", "gemm_reference"]
