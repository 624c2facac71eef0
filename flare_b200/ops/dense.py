"""Dense-tower ops: dot interaction, fused head + BCE, casts, initialisers.

CUDA tensors run the hand-written sm_100a kernels; CPU tensors run the fp32
reference implementations defined here (used as numerics oracles and by the
CPU configuration).
"""
from __future__ import annotations

import torch

from .._native import dtype_code, native, on_cuda


def interaction_pairs(num_vectors: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Index pairs (i > j) in the order the kernels emit them: row by row."""
    ii, jj = [], []
    for i in range(1, num_vectors):
        for j in range(i):
            ii.append(i)
            jj.append(j)
    return torch.tensor(ii, dtype=torch.long), torch.tensor(jj, dtype=torch.long)


def interaction_out_width(num_features: int, dim: int, pad_to: int = 16) -> int:
    t = num_features + 1
    w = dim + t * (t - 1) // 2
    return (w + pad_to - 1) // pad_to * pad_to


def interaction_forward(bot: torch.Tensor, emb: torch.Tensor, num_features: int, out: torch.Tensor,
                        status=None) -> torch.Tensor:
    """out[b] = [bot[b], <z_i, z_j> for i > j, zeros]  with z = [bot, emb_0..emb_{F-1}].

    On the GPU (up to 31 embedded features) four samples share one 128-row tcgen05 tile; ``status``
    (a ``DeviceStatus``) receives a timed-out tensor-core wait."""
    B, D = bot.shape
    if not on_cuda(bot, emb, out):
        z = torch.cat([bot.float().unsqueeze(1), emb.float().reshape(B, num_features, D)], dim=1)
        zz = torch.bmm(z, z.transpose(1, 2))
        ii, jj = interaction_pairs(num_features + 1)
        dots = zz[:, ii, jj]
        res = torch.zeros(out.shape, dtype=torch.float32)
        res[:, :D] = bot.float()
        res[:, D : D + dots.shape[1]] = dots
        out.copy_(res.to(out.dtype))
        return out
    native().interaction_forward(
        dict(B=B, F=num_features, D=D, bot=bot.data_ptr(), bot_ld=bot.stride(0), emb=emb.data_ptr(),
             emb_ld=emb.stride(0), out=out.data_ptr(), out_ld=out.stride(0),
             status=status.ptr if status is not None else 0)
    )
    return out


def interaction_backward(
    dout: torch.Tensor,
    bot: torch.Tensor,
    emb: torch.Tensor,
    num_features: int,
    dbot: torch.Tensor,
    demb: torch.Tensor,
    relu_mask_bot: bool = True,
    status=None,
) -> None:
    B, D = bot.shape
    if not on_cuda(dout, bot, emb, dbot, demb):
        t = num_features + 1
        z = torch.cat([bot.float().unsqueeze(1), emb.float().reshape(B, num_features, D)], dim=1)
        ii, jj = interaction_pairs(t)
        S = torch.zeros(B, t, t)
        g = dout.float()[:, D : D + ii.numel()]
        S[:, ii, jj] = g
        S[:, jj, ii] = g
        dz = torch.bmm(S, z)
        db = dz[:, 0] + dout.float()[:, :D]
        if relu_mask_bot:
            db = torch.where(bot.float() > 0, db, torch.zeros_like(db))
        dbot.copy_(db.to(dbot.dtype))
        demb.copy_(dz[:, 1:].reshape(B, num_features * D).to(demb.dtype))
        return
    native().interaction_backward(
        dict(B=B, F=num_features, D=D, bot=bot.data_ptr(), bot_ld=bot.stride(0), emb=emb.data_ptr(),
             emb_ld=emb.stride(0), dout=dout.data_ptr(), out_ld=dout.stride(0), dbot=dbot.data_ptr(),
             dbot_ld=dbot.stride(0), demb=demb.data_ptr(), demb_ld=demb.stride(0),
             relu_mask_bot=1 if relu_mask_bot else 0, status=status.ptr if status is not None else 0)
    )


def head_bce(
    h: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor,
    labels: torch.Tensor,
    *,
    grad_scale: float,
    logits: torch.Tensor,
    loss_sum: torch.Tensor,
    dh: torch.Tensor,
    dw: torch.Tensor,
    db: torch.Tensor,
    target_weights: torch.Tensor | None = None,
    sample_weights: torch.Tensor | None = None,
    valid_count: int = -1,
) -> None:
    """Fused prediction head + multi-target weighted sigmoid BCE, fwd + bwd.

    logits = h @ w.T + bias; loss_sum += sum(weight * BCE(logits, labels));
    dh = (dlogits @ w) * (h > 0); dw += dlogits.T @ h; db += dlogits.sum(0);
    dlogits = weight * (sigmoid(logits) - labels) * grad_scale.
    Semantics follow the reference's MultiTargetCrossEntropyLoss
    (recipes/recsys/ranking/losses.py:69-95) with sample weights and a valid
    prefix mask (recipes/recsys/ranking/graph/losses.py:29-40).
    """
    B, H = h.shape
    T = w.shape[0]
    lab = labels.reshape(B, -1)
    if not on_cuda(h, w, bias, labels, logits, loss_sum, dh, dw, db):
        hf = h.float()
        x = hf @ w.float().t() + bias.float()  # w, bias: compute copies
        y = lab.float()[:, :T]
        wt = torch.ones_like(x)
        if target_weights is not None:
            wt = wt * target_weights.float()
        if sample_weights is not None:
            wt = wt * sample_weights.float().reshape(B, 1)
        if valid_count >= 0:
            wt[valid_count:] = 0
        loss = torch.nn.functional.binary_cross_entropy_with_logits(x, y, reduction="none")
        loss_sum += (wt * loss).sum()
        dl = wt * (torch.sigmoid(x) - y) * grad_scale
        logits.copy_(x)
        dhv = dl @ w.float()
        dh.copy_(torch.where(hf > 0, dhv, torch.zeros_like(dhv)).to(dh.dtype))
        dw += dl.t() @ hf
        db += dl.sum(0)
        return
    native().head_bce(
        dict(B=B, H=H, T=T, h=h.data_ptr(), h_ld=h.stride(0), w=w.data_ptr(), bias=bias.data_ptr(),
             labels=labels.data_ptr(), label_ld=lab.stride(0),
             target_weights=target_weights.data_ptr() if target_weights is not None else 0,
             sample_weights=sample_weights.data_ptr() if sample_weights is not None else 0,
             valid_count=int(valid_count), grad_scale=float(grad_scale), logits=logits.data_ptr(),
             loss_sum=loss_sum.data_ptr(), dh=dh.data_ptr(), dh_ld=dh.stride(0), dw=dw.data_ptr(),
             db=db.data_ptr())
    )


def colsum_(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out += x.sum(0) for a bf16 [rows, cols] matrix, fp32 accumulation."""
    if not on_cuda(x, out):
        out += x.float().sum(0)
        return out
    native().colsum_bf16(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), out.data_ptr())
    return out


def cast_pad_bf16(x: torch.Tensor, out: torch.Tensor, *, zero: torch.Tensor | None = None) -> torch.Tensor:
    """out[:, :k] = bf16(x); out[:, k:] = 0; ``zero`` (an fp32 scalar, e.g. a step's loss accumulator) is
    cleared by the same launch."""
    if not on_cuda(x, out):
        out.zero_()
        out[:, : x.shape[1]] = x.to(out.dtype)
        if zero is not None:
            zero.zero_()
        return out
    if zero is not None and (zero.dtype != torch.float32 or not zero.is_cuda):
        raise ValueError("zero must be a CUDA fp32 tensor")
    native().cast_pad_bf16(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), out.data_ptr(), out.stride(0),
                           zero.data_ptr() if zero is not None else 0)
    return out


def init_uniform_(t: torch.Tensor, lo: float, hi: float, seed: int, index_offset: int = 0, *,
                  ncols: int | None = None, dim: int | None = None, col_begin: int = 0, row_stride: int = 1,
                  row_first: int = 0) -> torch.Tensor:
    """Fill ``t`` with uniform values from a counter-based generator.

    Value i of the stream depends only on (seed, index).  For a column slice
    (``t`` viewed as [rows, ncols] holding columns [col_begin, col_begin+ncols)
    of a table with row length ``dim``) element (r, c) takes stream index
    ``r*dim + col_begin + c``, so column shards reproduce the whole table.
    A row-wise piece holding table rows ``row_first + r*row_stride`` passes
    those two numbers and reproduces its rows of the whole table too.
    """
    if not t.is_contiguous():
        raise ValueError("init_uniform_ needs a contiguous tensor")
    n = t.numel()
    ncols = ncols or n
    dim = dim or ncols
    if not t.is_cuda:
        r = torch.arange(n) // ncols
        idx = (row_first + r * row_stride) * dim + col_begin + (torch.arange(n) - r * ncols) + index_offset
        t.copy_(uniform_at(idx, lo, hi, seed).reshape(t.shape).to(t.dtype))
        return t
    native().init_uniform(t.data_ptr(), dtype_code(t.dtype), n, float(lo), float(hi), int(seed),
                          int(index_offset), int(ncols), int(dim), int(col_begin), int(row_stride), int(row_first))
    return t


_M64 = (1 << 64) - 1


def _mix64(z: torch.Tensor) -> torch.Tensor:
    # splitmix64 finaliser on uint64 represented in int64 (wrapping arithmetic)
    z = z ^ (z >> 30 & ((1 << 34) - 1))
    z = z * torch.tensor(0xBF58476D1CE4E5B9 - (1 << 64), dtype=torch.int64)
    z = z ^ (z >> 27 & ((1 << 37) - 1))
    z = z * torch.tensor(0x94D049BB133111EB - (1 << 64), dtype=torch.int64)
    z = z ^ (z >> 31 & ((1 << 33) - 1))
    return z


def uniform_at(idx: torch.Tensor, lo: float, hi: float, seed: int) -> torch.Tensor:
    golden = 0x9E3779B97F4A7C15
    base = (seed * golden) & _M64
    if base >= 1 << 63:
        base -= 1 << 64
    z = _mix64(idx.to(torch.int64) + base)
    top24 = (z >> 40) & ((1 << 24) - 1)
    u = top24.to(torch.float64) / 16777216.0
    return (lo + (hi - lo) * u).to(torch.float32)


def uniform_reference(n: int, lo: float, hi: float, seed: int, index_offset: int = 0) -> torch.Tensor:
    return uniform_at(torch.arange(index_offset, index_offset + n, dtype=torch.int64), lo, hi, seed)


__all__ = [
    "cast_pad_bf16",
    "colsum_",
    "head_bce",
    "init_uniform_",
    "interaction_backward",
    "interaction_forward",
    "interaction_out_width",
    "interaction_pairs",
    "uniform_at",
    "uniform_reference",
]
