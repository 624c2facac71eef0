"""MLP tower on tcgen05 GEMMs with fused epilogues (explicit forward/backward).

Forward per layer: ``y = relu(x @ W.T + b)`` in one GEMM (bias + ReLU in the
epilogue).  Backward walks the layers once:

* ``dW += g.T @ x`` - one GEMM with both operands MN-major (no transposes),
  accumulated in fp32 straight into the flat gradient buffer;
* ``g_prev = (g @ W) * (x > 0)`` - one GEMM whose epilogue applies the
  previous layer's ReLU backward and accumulates ``db_prev`` (column sums).

Activation buffers are allocated once per batch size, so a whole training
step can be captured in a CUDA graph.  Mirrors the reference's MLP layer
(src/flare/jax/layers/base.py:27) semantically.
"""
from __future__ import annotations

import math

import torch

from ..ops.dense import colsum_
from ..ops.gemm import gemm
from ..training.flat import DenseState, FlatParams


def pad_to(n: int, m: int = 16) -> int:
    return (n + m - 1) // m * m


class MLPTower:
    def __init__(self, name: str, dims: list[int], params: FlatParams, *, relu_last: bool = True,
                 in_features: int | None = None):
        if len(dims) < 2:
            raise ValueError("an MLP needs an input and at least one layer width")
        self.name = name
        self.dims = [pad_to(dims[0])] + [int(d) for d in dims[1:]]
        self.true_in = in_features if in_features is not None else dims[0]
        for d in self.dims[1:]:
            if d % 16:
                raise ValueError(f"hidden width {d} must be a multiple of 16")
        self.relu = [True] * (len(self.dims) - 2) + [relu_last]
        self.wnames, self.bnames = [], []
        for i in range(len(self.dims) - 1):
            fan_in, fan_out = self.dims[i], self.dims[i + 1]
            wn, bn = f"{name}.{i}.weight", f"{name}.{i}.bias"
            # DLRM-style init: W ~ N(0, 2/(fan_in+fan_out)), b ~ N(0, 1/fan_out)
            params.register(wn, (fan_out, fan_in), "normal", math.sqrt(2.0 / (fan_in + fan_out)),
                            zero_cols_from=self.true_in if i == 0 and self.true_in < fan_in else None)
            params.register(bn, (fan_out,), "normal", math.sqrt(1.0 / fan_out))
            self.wnames.append(wn)
            self.bnames.append(bn)
        self.state: DenseState | None = None

    @property
    def out_dim(self) -> int:
        return self.dims[-1]

    @property
    def in_dim(self) -> int:
        return self.dims[0]

    def bind(self, state: DenseState, batch: int) -> None:
        """Attach parameter views and allocate activation/gradient buffers."""
        self.state = state
        dev = state.device
        self.W = [state.compute_view(n) for n in self.wnames]
        self.b = [state.compute_view(n) for n in self.bnames]
        self.dW = [state.grad_view(n) for n in self.wnames]
        self.db = [state.grad_view(n) for n in self.bnames]
        self.acts = [torch.empty(batch, d, dtype=torch.bfloat16, device=dev) for d in self.dims[1:]]
        self.grads = [torch.empty(batch, d, dtype=torch.bfloat16, device=dev) for d in self.dims[:-1]]
        self.x = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self.x = x
        h = x
        for i in range(len(self.W)):
            gemm(h, self.W[i], bias=self.b[i], relu=self.relu[i], out=self.acts[i])
            h = self.acts[i]
        return h

    def backward(self, g_pre: torch.Tensor, *, need_input_grad: bool = False,
                 input_mask: torch.Tensor | None = None) -> torch.Tensor | None:
        """``g_pre``: gradient w.r.t. the last layer's pre-activation (already ReLU-masked)."""
        L = len(self.W)
        colsum_(g_pre, self.db[L - 1])
        g = g_pre
        for i in range(L - 1, -1, -1):
            xin = self.x if i == 0 else self.acts[i - 1]
            gemm(g, xin, a_t=True, b_t=True, out=self.dW[i], accumulate=True)
            if i > 0:
                gemm(g, self.W[i], b_t=True, out=self.grads[i], mask=self.acts[i - 1] if self.relu[i - 1] else None,
                     colsum=self.db[i - 1])
                g = self.grads[i]
            elif need_input_grad:
                gemm(g, self.W[0], b_t=True, out=self.grads[0], mask=input_mask)
                return self.grads[0]
        return None

    def flops_per_sample(self) -> int:
        return sum(2 * self.dims[i] * self.dims[i + 1] for i in range(len(self.dims) - 1))


__all__ = ["MLPTower", "pad_to"]
