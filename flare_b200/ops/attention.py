"""Jagged causal multi-head attention (8 heads x 32) on tcgen05, with a PyTorch reference.

Tokens of many sequences are packed into one ``[T_cap, ...]`` matrix; sequence
``s`` occupies rows ``offsets[s] .. offsets[s+1]``; every sequence is padded at
its end to a multiple of 8 tokens (``pack_offsets``), so TMA coordinates along
the token axis stay 16-byte aligned.  Rows after ``offsets[-1]`` are ignored.

``AttentionBuffers`` holds the static buffers of one layer (so a training step
is CUDA-graph capturable): QKV ``[T_cap, 768]``, V^T / Q^T / dO^T ``[256, T_cap]``,
output, log-sum-exp, the backward workspaces and dQKV.
"""
from __future__ import annotations

import math

import torch

from .._native import DEFAULT_TIMEOUT_NS, DeviceStatus, native

HEADS, HEAD_DIM = 8, 32
DMODEL = HEADS * HEAD_DIM


def pack_offsets(lengths: list[int] | torch.Tensor, align: int = 8) -> tuple[torch.Tensor, torch.Tensor]:
    """(offsets [n+1], valid [offsets[-1]]) for sequences padded at their END to a multiple of ``align``.

    Padding tokens sit after the real ones, so causal attention never lets a
    real token see them; the caller gives them zero loss gradient, which makes
    their backward contributions vanish as well.
    """
    lens = [int(x) for x in (lengths.tolist() if isinstance(lengths, torch.Tensor) else lengths)]
    offs = [0]
    for L in lens:
        offs.append(offs[-1] + (L + align - 1) // align * align)
    valid = torch.zeros(offs[-1], dtype=torch.bool)
    for s, L in enumerate(lens):
        valid[offs[s]:offs[s] + L] = True
    return torch.tensor(offs, dtype=torch.int32), valid


def jagged_attention_reference(qkv: torch.Tensor, offsets: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """fp32 causal attention per sequence and head (the numerics oracle)."""
    scale = scale or 1.0 / math.sqrt(HEAD_DIM)
    T = qkv.shape[0]
    out = torch.zeros(T, DMODEL, dtype=torch.float32, device=qkv.device)
    offs = offsets.tolist()
    x = qkv.float()
    for s in range(len(offs) - 1):
        a, b = offs[s], offs[s + 1]
        if b <= a:
            continue
        L = b - a
        q = x[a:b, :DMODEL].view(L, HEADS, HEAD_DIM).transpose(0, 1)
        k = x[a:b, DMODEL:2 * DMODEL].view(L, HEADS, HEAD_DIM).transpose(0, 1)
        v = x[a:b, 2 * DMODEL:3 * DMODEL].view(L, HEADS, HEAD_DIM).transpose(0, 1)
        att = (q @ k.transpose(1, 2)) * scale
        mask = torch.ones(L, L, dtype=torch.bool, device=qkv.device).tril()
        att = att.masked_fill(~mask, float("-inf")).softmax(-1)
        out[a:b] = (att @ v).transpose(0, 1).reshape(L, DMODEL)
    return out


class AttentionBuffers:
    """Static per-layer buffers for the fused forward/backward."""

    def __init__(self, T_cap: int, device: torch.device):
        if T_cap % 8:
            raise ValueError("token capacity must be a multiple of 8")
        self.T_cap = T_cap
        bf = dict(dtype=torch.bfloat16, device=device)
        self.qkv = torch.zeros(T_cap, 3 * DMODEL, **bf)
        self.vt = torch.zeros(DMODEL, T_cap, **bf)
        self.qt = torch.zeros(DMODEL, T_cap, **bf)
        self.out = torch.zeros(T_cap, DMODEL, **bf)
        self.lse = torch.zeros(HEADS, T_cap, dtype=torch.float32, device=device)
        self.dout = torch.zeros(T_cap, DMODEL, **bf)
        self.dout_t = torch.zeros(DMODEL, T_cap, **bf)
        self.delta = torch.zeros(HEADS, T_cap, dtype=torch.float32, device=device)
        self.dq_acc = torch.zeros(T_cap, DMODEL, dtype=torch.float32, device=device)
        self.dqkv = torch.zeros(T_cap, 3 * DMODEL, **bf)
        self.status = DeviceStatus(device)


def jagged_attention_forward(buf: AttentionBuffers, offsets: torch.Tensor, nseq: int, max_len: int,
                             scale: float | None = None) -> torch.Tensor:
    """out = attention(buf.qkv) using buf.vt (V^T, filled by the caller); returns buf.out."""
    native().attn_forward(dict(
        qkv=buf.qkv.data_ptr(), ld_qkv=buf.qkv.stride(0), vt=buf.vt.data_ptr(), ld_vt=buf.vt.stride(0),
        offsets=offsets.data_ptr(), nseq=int(nseq), max_len=int(max_len), T_cap=buf.T_cap,
        scale=float(scale or 1.0 / math.sqrt(HEAD_DIM)), out=buf.out.data_ptr(), ld_out=buf.out.stride(0),
        lse=buf.lse.data_ptr(), ld_lse=buf.lse.stride(0), status=buf.status.ptr, timeout_ns=DEFAULT_TIMEOUT_NS))
    return buf.out


def jagged_attention_backward(buf: AttentionBuffers, offsets: torch.Tensor, nseq: int, max_len: int,
                              scale: float | None = None) -> torch.Tensor:
    """dQKV from buf.dout / buf.dout_t (filled by the caller) and buf.qt (Q^T); returns buf.dqkv."""
    native().attn_backward(dict(
        qkv=buf.qkv.data_ptr(), ld_qkv=buf.qkv.stride(0), dout=buf.dout.data_ptr(), out=buf.out.data_ptr(),
        ld_do=buf.dout.stride(0), dout_t=buf.dout_t.data_ptr(), q_t=buf.qt.data_ptr(), ld_t=buf.qt.stride(0),
        offsets=offsets.data_ptr(), nseq=int(nseq), max_len=int(max_len), T_cap=buf.T_cap,
        scale=float(scale or 1.0 / math.sqrt(HEAD_DIM)), lse=buf.lse.data_ptr(), delta=buf.delta.data_ptr(),
        ld_stat=buf.lse.stride(0), dq_acc=buf.dq_acc.data_ptr(), ld_dq=buf.dq_acc.stride(0),
        dqkv=buf.dqkv.data_ptr(), ld_dqkv=buf.dqkv.stride(0), status=buf.status.ptr,
        timeout_ns=DEFAULT_TIMEOUT_NS))
    return buf.dqkv


__all__ = ["AttentionBuffers", "DMODEL", "HEADS", "HEAD_DIM", "jagged_attention_backward", "jagged_attention_forward",
           "jagged_attention_reference", "pack_offsets"]
