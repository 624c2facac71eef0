"""Fused multitask-layer ops: expert mixing through a gate and the MLP ReLU backward.

``gate_mix(logits, experts)`` returns ``sum_e softmax(logits)_e * experts[e]``
(fp32 softmax and accumulation, bf16 out) as one autograd node: the forward
reads every expert row once and the backward writes every expert gradient
and the gate-logit gradient in one more pass (``csrc/mixing.cu``).  It
replaces the stack / softmax / multiply / sum sequence of the reference's
``_mix`` (src/flare/jax/layers/multitask.py) on bf16 CUDA tensors; anything
else takes the eager path.

``relu_bwd_colsum_(g, h, out, colsum)``: ``out = g * (h > 0)`` and
``colsum += out.sum(0)`` in one pass (the ReLU backward of an MLP layer with
its bias gradient).
"""
from __future__ import annotations

import torch

from .._native import native, on_cuda

MAX_EXPERTS = 64
MAX_WIDTH = 1024


def _aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0 and t.stride(-1) == 1 and t.stride(0) % 8 == 0


def gate_mix_supported(logits: torch.Tensor, experts: list[torch.Tensor]) -> bool:
    if not experts or len(experts) > MAX_EXPERTS or logits.dim() != 2 or logits.shape[1] != len(experts):
        return False
    y0 = experts[0]
    if not (logits.is_cuda and logits.dtype == torch.bfloat16 and logits.stride(1) == 1):
        return False
    if y0.dim() != 2 or y0.shape[0] != logits.shape[0] or y0.shape[1] % 8 or y0.shape[1] > MAX_WIDTH:
        return False
    return all(y.is_cuda and y.dtype == torch.bfloat16 and y.shape == y0.shape and y.stride() == y0.stride()
               and _aligned(y) for y in experts)


class _GateMixFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, *ys):
        B, E = logits.shape
        D = ys[0].shape[1]
        out = torch.empty(B, D, dtype=torch.bfloat16, device=logits.device)
        probs = torch.empty(B, E, dtype=torch.float32, device=logits.device)
        native().gate_mix(dict(ys=[y.data_ptr() for y in ys], logits=logits.data_ptr(), ld_logits=logits.stride(0),
                               probs=probs.data_ptr(), ld_y=ys[0].stride(0), ld_out=D, B=B, D=D,
                               out=out.data_ptr()), False)
        ctx.save_for_backward(probs, *ys)
        return out

    @staticmethod
    def backward(ctx, dout):
        probs, *ys = ctx.saved_tensors
        B, E = probs.shape
        D = ys[0].shape[1]
        dout = dout.to(torch.bfloat16).contiguous()
        dys = [torch.empty(B, D, dtype=torch.bfloat16, device=dout.device) for _ in ys]
        dlogits = torch.empty(B, E, dtype=torch.bfloat16, device=dout.device)
        # the backward reads the saved probabilities, not the logits
        native().gate_mix(dict(ys=[y.data_ptr() for y in ys], logits=dlogits.data_ptr(), ld_logits=E,
                               probs=probs.data_ptr(), ld_y=ys[0].stride(0), ld_out=D, B=B, D=D,
                               dys=[d.data_ptr() for d in dys], ld_dy=D, dlogits=dlogits.data_ptr(),
                               dout=dout.data_ptr()), True)
        return (dlogits, *dys)


def gate_mix_reference(logits: torch.Tensor, experts: list[torch.Tensor]) -> torch.Tensor:
    """fp32 softmax and sum, cast to the experts' dtype (the eager path)."""
    p = torch.softmax(logits.float(), -1)
    return (torch.stack([y.float() for y in experts], -1) * p.unsqueeze(1)).sum(-1).to(experts[0].dtype)


def gate_mix(logits: torch.Tensor, experts: list[torch.Tensor]) -> torch.Tensor:
    if gate_mix_supported(logits, experts):
        return _GateMixFn.apply(logits, *experts)
    return gate_mix_reference(logits, experts)


def relu_bwd_colsum_(g: torch.Tensor, h: torch.Tensor, out: torch.Tensor, colsum: torch.Tensor) -> torch.Tensor:
    if not on_cuda(g, h, out, colsum):
        out.copy_(torch.where(h > 0, g, torch.zeros_like(g)))
        colsum += out.float().sum(0)
        return out
    native().relu_bwd_colsum(g.data_ptr(), g.stride(0), h.data_ptr(), h.stride(0), g.shape[0], g.shape[1],
                             out.data_ptr(), out.stride(0), colsum.data_ptr())
    return out


__all__ = ["gate_mix", "gate_mix_reference", "gate_mix_supported", "relu_bwd_colsum_"]
