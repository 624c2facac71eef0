"""Dense layer library (PyTorch modules).

Same constructor contracts and semantics as the reference's layer library
(src/flare/jax/layers/__init__.py:3-21): ``MLP``; ``CategoricalEmbedding``
(side-information tables grouped by dim, sum/mean pooling with id 0 as null,
fp32 tables); the multitask gates ``PLE`` / ``CGC`` / ``UPLE`` / ``UCGC``;
``TokenMix``; ``BatchedExpertMoE`` (dense or top-k soft gating, SwiGLU
experts, RMS-normalised residual); the multi-head MoE token mixers
``TokenMixLargeMoe`` / ``TokenMixLargePreGateNoPool``; ``NamedTokens``; fp32
numerics helpers.

``TcLinear`` is a linear layer whose forward and backward GEMMs run on the
hand-written tcgen05 kernel when the input is a bf16 CUDA tensor (weight
gradients accumulate in fp32, as ``fp32_weight_gradient_dot_general`` does in
the reference); otherwise it is a plain fp32 ``nn.Linear``.  A ReLU ``MLP`` on
bf16 CUDA inputs runs as one autograd node: bias + ReLU in the GEMM
epilogues, and in the backward each layer's input-gradient GEMM applies the
previous layer's ReLU mask and sums its bias gradient in the epilogue.  The
gates' expert mixing is one fused kernel per direction (``ops.mixing``).
"""
from __future__ import annotations

import math
from collections.abc import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.dense import colsum_
from ..ops.gemm import gemm
from ..ops.mixing import gate_mix, relu_bwd_colsum_


# ---------------------------------------------------------------- numerics
def fp32_softmax(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    return torch.softmax(x.float(), dim=dim).to(x.dtype)


def fp32_mean(x: torch.Tensor, dim=None, keepdim: bool = False) -> torch.Tensor:
    out = x.float().mean() if dim is None else x.float().mean(dim=dim, keepdim=keepdim)
    return out.to(x.dtype)


def fp32_sum(x: torch.Tensor, dim=None, keepdim: bool = False) -> torch.Tensor:
    out = x.float().sum() if dim is None else x.float().sum(dim=dim, keepdim=keepdim)
    return out.to(x.dtype)


def fp32_rms_normalize(x: torch.Tensor, dim: int = -1, eps: float = 1e-5) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=dim, keepdim=True) + eps)).to(x.dtype)


# ----------------------------------------------------------- tcgen05 linear
class _TcLinearFn(torch.autograd.Function):
    """y = x W^T + b on the tcgen05 GEMM.  A weight bound to a flat fused optimizer (it carries
    ``_flare_grad``, an fp32 view of the flat gradient buffer) receives ``dW`` straight from the GEMM
    epilogue (accumulated in fp32) and its bias ``db`` from a column-sum kernel; autograd then gets no
    gradient for them.  An unbound weight gets an ordinary fp32 gradient."""

    @staticmethod
    def forward(ctx, x, w, b):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        wb = w.to(torch.bfloat16).contiguous()
        bb = b.to(torch.bfloat16) if b is not None else None
        y = gemm(x2, wb, bias=bb)
        ctx.save_for_backward(x2, wb)
        ctx.has_bias = b is not None
        ctx.shape = x.shape
        ctx.flat_w = getattr(w, "_flare_grad", None)
        ctx.flat_b = getattr(b, "_flare_grad", None) if b is not None else None
        return y.reshape(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, wb = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1]).to(torch.bfloat16).contiguous()
        dx = gemm(g2, wb, b_t=True).reshape(ctx.shape) if ctx.needs_input_grad[0] else None
        dw = db = None
        if ctx.flat_w is not None:
            gemm(g2, x2, a_t=True, b_t=True, out=ctx.flat_w, accumulate=True)
        elif ctx.needs_input_grad[1]:
            dw = torch.zeros(wb.shape, dtype=torch.float32, device=wb.device)
            gemm(g2, x2, a_t=True, b_t=True, out=dw, accumulate=True)
        if ctx.has_bias:
            if ctx.flat_b is not None:
                colsum_(g2, ctx.flat_b)
            elif ctx.needs_input_grad[2]:
                db = g2.float().sum(0)
        return dx, dw, db


class TcLinear(nn.Linear):
    """nn.Linear that uses the tcgen05 GEMM for bf16 CUDA inputs (dims multiple of 8)."""

    def tc_eligible(self, x: torch.Tensor) -> bool:
        return x.is_cuda and x.dtype == torch.bfloat16 and self.in_features % 8 == 0 and self.out_features % 8 == 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tc_eligible(x):
            return _TcLinearFn.apply(x, self.weight, self.bias)
        return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))


class _TcReluMLPFn(torch.autograd.Function):
    """A stack of TcLinear layers with ReLU between them (and optionally after the last) as one node.

    Forward: bias + ReLU in every GEMM epilogue.  Backward: the last layer's ReLU mask and bias
    gradient in one pass (``relu_bwd_colsum``); then per layer the weight gradient (fp32, accumulated
    into the flat buffer when bound) and the input-gradient GEMM whose epilogue applies the previous
    layer's ReLU mask and adds the previous layer's bias gradient."""

    @staticmethod
    def forward(ctx, x, last_relu, *params):
        L = len(params) // 2
        h = x.reshape(-1, x.shape[-1]).contiguous()
        hs, wbs = [h], []
        for i in range(L):
            w, b = params[2 * i], params[2 * i + 1]
            wb = w.to(torch.bfloat16).contiguous()
            h = gemm(h, wb, bias=b.to(torch.bfloat16), relu=i < L - 1 or last_relu)
            hs.append(h)
            wbs.append(wb)
        ctx.save_for_backward(*hs, *wbs)
        ctx.L, ctx.last_relu, ctx.shape = L, last_relu, x.shape
        ctx.flat = [getattr(p, "_flare_grad", None) for p in params]
        ctx.param_shapes = [p.shape for p in params]
        return h.reshape(*x.shape[:-1], h.shape[-1])

    @staticmethod
    def backward(ctx, gy):
        L = ctx.L
        saved = ctx.saved_tensors
        hs, wbs = saved[:L + 1], saved[L + 1:]
        dev = gy.device
        grads: list[torch.Tensor | None] = [None] * (2 * L)

        def target(k):  # where parameter k's gradient goes: its flat fp32 view, or a fresh fp32 buffer
            if ctx.flat[k] is not None:
                return ctx.flat[k]
            grads[k] = torch.zeros(ctx.param_shapes[k], dtype=torch.float32, device=dev)
            return grads[k]

        g = gy.reshape(-1, gy.shape[-1]).to(torch.bfloat16).contiguous()
        db = target(2 * L - 1)
        if ctx.last_relu:
            gm = torch.empty_like(g)
            relu_bwd_colsum_(g, hs[L], gm, db)
            g = gm
        else:
            colsum_(g, db)
        dx = None
        for i in reversed(range(L)):
            gemm(g, hs[i], a_t=True, b_t=True, out=target(2 * i), accumulate=True)
            if i > 0:
                g = gemm(g, wbs[i], b_t=True, mask=hs[i], colsum=target(2 * i - 1))
            elif ctx.needs_input_grad[0]:
                dx = gemm(g, wbs[0], b_t=True).reshape(ctx.shape)
        return (dx, None, *grads)


_ACTS = {"relu": F.relu, "gelu": F.gelu, "sigmoid": torch.sigmoid, "tanh": torch.tanh,
         "softmax": lambda x: fp32_softmax(x, -1)}


def get_activation(name: str | None):
    if name is None or name.lower() == "none":
        return None
    try:
        return _ACTS[name.lower()]
    except KeyError as exc:
        raise ValueError(f"unsupported activation: {name!r}") from exc


def _stacked_view(params, attr: str | None, rows: int, cols: int) -> torch.Tensor | None:
    """One [rows, cols] view over consecutive equal-shaped tensors (``p.data`` or ``p.<attr>``), or None when
    they are not laid out back to back (flat-buffer parameters registered as a stack group are)."""
    ts = [getattr(p, attr, None) if attr else p.data for p in params]
    if any(t is None for t in ts):
        return None
    t0 = ts[0]
    n = t0.numel()
    es = t0.element_size()
    base = t0.untyped_storage()
    if (t0.storage_offset() + rows * cols) * es > base.nbytes():
        return None  # separate allocations that merely sit next to each other are not one buffer
    for k, t in enumerate(ts):
        if t.dtype != t0.dtype or t.numel() != n or not t.is_contiguous() or \
                t.untyped_storage().data_ptr() != base.data_ptr() or t.data_ptr() != t0.data_ptr() + k * n * es:
            return None
    return t0.as_strided((rows, cols), (cols, 1))


class _StackedReluLinearFn(torch.autograd.Function):
    """n single-layer experts on one input as one GEMM: y = x [W_0; ...; W_{n-1}]^T + [b_0; ...] (ReLU
    optional), returned as n column views.  Experts whose parameters sit back to back in the flat fused
    buffers (a stack group of ``FusedDenseParameters``) use those buffers directly: no weight copy in the
    forward, and the weight / bias gradients land in the flat gradient buffer from the GEMM epilogue and
    the ReLU-backward column sums."""

    @staticmethod
    def forward(ctx, x, last_relu, n, *params):
        Ws, bs = params[:n], params[n:]
        D, K = Ws[0].shape
        x2 = x.reshape(-1, K).contiguous()
        wc = _stacked_view(Ws, None, n * D, K)
        if wc is None or wc.dtype != torch.bfloat16:
            wc = torch.cat([w.to(torch.bfloat16) for w in Ws])
        bc = _stacked_view(bs, None, 1, n * D)
        bc = bc.reshape(-1) if bc is not None and bc.dtype == torch.bfloat16 else torch.cat(
            [b.to(torch.bfloat16) for b in bs])
        y = gemm(x2, wc, bias=bc, relu=bool(last_relu))
        ctx.save_for_backward(x2, wc, y)
        ctx.n, ctx.D, ctx.K, ctx.last_relu, ctx.shape = n, D, K, bool(last_relu), x.shape
        ctx.params = params
        return tuple(y[:, e * D:(e + 1) * D].reshape(*x.shape[:-1], D) for e in range(n))

    @staticmethod
    def backward(ctx, *gys):
        x2, wc, y = ctx.saved_tensors
        n, D, K = ctx.n, ctx.D, ctx.K
        Ws, bs = ctx.params[:n], ctx.params[n:]
        dev = y.device
        g = torch.cat([(gy if gy is not None else torch.zeros(y.shape[0], D, device=dev)).reshape(-1, D)
                       .to(torch.bfloat16) for gy in gys], 1)
        dw = _stacked_view(Ws, "_flare_grad", n * D, K)
        db = _stacked_view(bs, "_flare_grad", 1, n * D)
        flat = dw is not None and db is not None
        if not flat:
            dw = torch.zeros(n * D, K, dtype=torch.float32, device=dev)
            db = torch.zeros(n * D, dtype=torch.float32, device=dev)
        db = db.reshape(-1)
        if ctx.last_relu:
            gm = torch.empty_like(g)
            relu_bwd_colsum_(g, y, gm, db)
            g = gm
        else:
            colsum_(g, db)
        gemm(g, x2, a_t=True, b_t=True, out=dw, accumulate=True)
        dx = gemm(g, wc, b_t=True).reshape(ctx.shape) if ctx.needs_input_grad[0] else None
        if flat:
            grads = [None] * (2 * n)
        else:
            grads = [dw[e * D:(e + 1) * D] for e in range(n)] + [db[e * D:(e + 1) * D] for e in range(n)]
        return (dx, None, None, *grads)


class MLP(nn.Module):
    def __init__(self, in_features: int, dims: Sequence[int], activate: str = "relu",
                 last_layer_use_activate: bool = True):
        super().__init__()
        self.layers = nn.ModuleList()
        for d in dims:
            self.layers.append(TcLinear(in_features, d))
            in_features = d
        self.dims = list(dims)
        self.activate = activate
        self.last_layer_use_activate = last_layer_use_activate

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if (self.activate is not None and str(self.activate).lower() == "relu" and self.layers
                and all(layer.bias is not None and layer.tc_eligible(x) for layer in self.layers)):
            params = [t for layer in self.layers for t in (layer.weight, layer.bias)]
            return _TcReluMLPFn.apply(x, self.last_layer_use_activate, *params)
        act = get_activation(self.activate)
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if act is not None and (i < len(self.layers) - 1 or self.last_layer_use_activate):
                x = act(x)
        return x


# ------------------------------------------------------- categorical embedding
class CategoricalEmbedding(nn.Module):
    """Dense side-information tables grouped by dim; id 0 is null (side-info +1 shift)."""

    def __init__(self, cate_feature_metas: dict[str, tuple[int, int]], side_info_layout: dict[str, tuple[int, int]],
                 pooling: str = "sum"):
        super().__init__()
        if pooling not in ("sum", "mean"):
            raise ValueError(f"Unsupported pooling method: {pooling}")
        self.pooling = pooling
        totals: dict[int, int] = {}
        self.vocab_offsets: dict[str, int] = {}
        groups: dict[tuple[int, int], list[str]] = {}
        for k, (vocab, dim) in cate_feature_metas.items():
            if k not in side_info_layout:
                raise ValueError(f"Feature {k!r} not found in side_info_layout")
            self.vocab_offsets[k] = totals.get(dim, 0)
            totals[dim] = totals.get(dim, 0) + vocab + 2
            groups.setdefault((dim, side_info_layout[k][1]), []).append(k)
        self.tables = nn.ParameterDict({str(d): nn.Parameter(torch.randn(n, d)) for d, n in totals.items()})
        self.meta = []
        for (dim, flen), keys in groups.items():
            idx = torch.tensor([[side_info_layout[k][0] + i for i in range(flen)] for k in keys])
            off = torch.tensor([self.vocab_offsets[k] for k in keys])
            self.register_buffer(f"idx_{dim}_{flen}", idx, persistent=False)
            self.register_buffer(f"off_{dim}_{flen}", off, persistent=False)
            self.meta.append((dim, flen, keys))
        self.feature_order = {d: [k for (dd, _, ks) in self.meta if dd == d for k in ks] for d in totals}

    def forward(self, side_info: torch.Tensor) -> dict[int, torch.Tensor]:
        out: dict[int, list[torch.Tensor]] = {}
        for dim, flen, _ in self.meta:
            idx = getattr(self, f"idx_{dim}_{flen}")
            off = getattr(self, f"off_{dim}_{flen}")
            ids = side_info[:, idx]                          # [B, K, flen]
            emb = self.tables[str(dim)].float()[ids + off.view(1, -1, 1)]
            if flen > 1:
                mask = (ids != 0).unsqueeze(-1)
                pooled = (emb * mask).sum(2)
                if self.pooling == "mean":
                    pooled = pooled / mask.sum(2).clamp_min(1)
            else:
                pooled = emb[:, :, 0]
            out.setdefault(dim, []).append(pooled)
        return {d: torch.cat(v, 1) for d, v in out.items()}


# ------------------------------------------------------------- multitask
class _GatedExperts(nn.Module):
    def __init__(self, base_dim, gate_in_dim, num_experts, dims, n_tasks, activate, gate_sizes):
        super().__init__()
        self.num_experts, self.n_tasks, self.out_dim = num_experts, n_tasks, dims[-1]
        self.experts = nn.ModuleList(MLP(base_dim, dims, activate) for _ in range(n_tasks * num_experts))
        self.gate_layers = nn.ModuleList(TcLinear(gate_in_dim, g) for g in gate_sizes)
        # single-layer ReLU experts are computed as one stacked GEMM per shared input; their weights
        # and biases form stack groups, which FusedDenseParameters lays out back to back
        self.stackable = len(dims) == 1 and str(activate).lower() == "relu" and dims[0] % 8 == 0 \
            and base_dim % 8 == 0
        if self.stackable:
            gid = id(self)
            for e, m in enumerate(self.experts):
                m.layers[0].weight._flare_stack = (gid, "w", e)
                m.layers[0].bias._flare_stack = (gid, "b", e)

    def _expert_outputs(self, base_layers):
        x0 = base_layers[0]
        if self.stackable and x0.is_cuda and x0.dtype == torch.bfloat16:
            # consecutive input groups that share one tensor run as one GEMM
            outs, i, t = [], 0, 0
            while t < len(base_layers):
                u = t
                while u + 1 < len(base_layers) and base_layers[u + 1] is base_layers[t]:
                    u += 1
                ex = [self.experts[k].layers[0] for k in range(i, i + (u - t + 1) * self.num_experts)]
                last = self.experts[i].last_layer_use_activate
                ys = _StackedReluLinearFn.apply(base_layers[t], last, len(ex), *[l.weight for l in ex],
                                                *[l.bias for l in ex])
                for k in range(u - t + 1):
                    outs.append(list(ys[k * self.num_experts:(k + 1) * self.num_experts]))
                i += (u - t + 1) * self.num_experts
                t = u + 1
            return outs
        outs, i = [], 0
        for t in range(len(base_layers)):
            outs.append([self.experts[i + e](base_layers[t]) for e in range(self.num_experts)])
            i += self.num_experts
        return outs

    @staticmethod
    def _mix(layers, gate_logits):
        if gate_logits.dim() == 2 and gate_logits.is_cuda and gate_logits.dtype == torch.bfloat16:
            return gate_mix(gate_logits, list(layers))  # one fused kernel per direction
        stacked = torch.stack(layers, -1)                     # [B, D, E]
        gate = fp32_softmax(gate_logits, -1).unsqueeze(1)     # [B, 1, E]
        return fp32_sum(stacked * gate, dim=-1)


class PLE(_GatedExperts):
    """Progressive layered extraction: N task inputs + 1 shared -> N+1 outputs."""

    def __init__(self, base_dim, gate_in_dim, num_experts, dims, n_tasks, activate="relu"):
        shared = n_tasks - 1
        super().__init__(base_dim, gate_in_dim, num_experts, dims, n_tasks, activate,
                         [num_experts * 2 if i != shared else num_experts * n_tasks for i in range(n_tasks)])

    def forward(self, base_layers, gate_layer):
        eo = self._expert_outputs(base_layers)
        shared = len(base_layers) - 1
        out = []
        for i in range(len(base_layers)):
            layers = eo[i] + eo[shared] if i != shared else [e for row in eo for e in row]
            out.append(self._mix(layers, self.gate_layers[i](gate_layer)))
        return out


class CGC(_GatedExperts):
    """Customized gate control: N task inputs + 1 shared -> N outputs."""

    def __init__(self, base_dim, gate_in_dim, num_experts, dims, n_tasks, activate="relu"):
        super().__init__(base_dim, gate_in_dim, num_experts, dims, n_tasks, activate,
                         [num_experts * 2] * (n_tasks - 1))

    def forward(self, base_layers, gate_layer):
        eo = self._expert_outputs(base_layers)
        shared = len(base_layers) - 1
        return [self._mix(eo[i] + eo[shared], self.gate_layers[i](gate_layer)) for i in range(len(base_layers) - 1)]


class UPLE(PLE):
    """PLE with a separate gate input per task."""

    def forward(self, base_layers, gate_layers_in):
        eo = self._expert_outputs(base_layers)
        shared = len(base_layers) - 1
        out = []
        for i in range(len(base_layers)):
            layers = eo[i] + eo[shared] if i != shared else [e for row in eo for e in row]
            out.append(self._mix(layers, self.gate_layers[i](gate_layers_in[i])))
        return out


class UCGC(CGC):
    """CGC with a separate gate input per task."""

    def forward(self, base_layers, gate_layers_in):
        eo = self._expert_outputs(base_layers)
        shared = len(base_layers) - 1
        return [self._mix(eo[i] + eo[shared], self.gate_layers[i](gate_layers_in[i]))
                for i in range(len(base_layers) - 1)]


# -------------------------------------------------------------- token mix
class TokenMix(nn.Module):
    """Slice-and-concat token mixing, LayerNorm, GELU FFN, LayerNorm, mean pooling."""

    def __init__(self, token_num: int, token_dim: int, layer_size: int, hidden_dims: Sequence[int] = ()):
        super().__init__()
        if token_dim % token_num:
            raise ValueError("token_dim must be divisible by token_num")
        self.token_num, self.token_dim, self.layer_size = token_num, token_dim, layer_size
        self.slice_dim = token_dim // token_num
        n = layer_size * token_num
        self.mix_lns = nn.ModuleList(nn.LayerNorm(token_dim, eps=1e-3) for _ in range(n))
        self.mix_ffns = nn.ModuleList(MLP(token_dim, list(hidden_dims) + [token_dim], activate="gelu")
                                      for _ in range(n))
        self.ffn_lns = nn.ModuleList(nn.LayerNorm(token_dim, eps=1e-3) for _ in range(n))

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        out = [tokens[:, j] for j in range(self.token_num)]
        idx = 0
        for _ in range(self.layer_size):
            mixed = [torch.cat([t[..., j * self.slice_dim:(j + 1) * self.slice_dim] for t in out], -1)
                     for j in range(self.token_num)]
            new = []
            for j in range(self.token_num):
                a = self.mix_lns[idx](out[j] + mixed[j])
                new.append(self.ffn_lns[idx](a + self.mix_ffns[idx](a)))
                idx += 1
            out = new
        return fp32_mean(torch.stack(out, 1), dim=1)


class BatchedExpertMoE(nn.Module):
    """Per-slot batched SwiGLU experts with dense or top-k softmax gating.

    Input ``x`` is [slots, batch, in_dim]; every slot has its own experts.
    """

    def __init__(self, batch_dim: int, in_dim: int, scale_size: int, num_experts: int, sparse: bool, top_k: int,
                 residual_norm: bool = True):
        super().__init__()
        self.batch_dim, self.in_dim, self.num_experts = batch_dim, in_dim, num_experts
        self.sparse, self.top_k, self.residual_norm = sparse, min(top_k, num_experts), residual_norm
        h = in_dim * scale_size
        lecun = lambda *s: torch.randn(*s) / math.sqrt(s[-2])  # noqa: E731
        if num_experts > 1:
            self.w_gate = nn.Parameter(lecun(batch_dim, in_dim, num_experts))
            self.b_gate = nn.Parameter(torch.zeros(batch_dim, num_experts))
        self.w_up = nn.Parameter(lecun(batch_dim, num_experts, in_dim, 2 * h))
        self.b_up = nn.Parameter(torch.zeros(batch_dim, num_experts, 2 * h))
        self.w_down = nn.Parameter(lecun(batch_dim, num_experts, h, in_dim))
        self.b_down = nn.Parameter(torch.zeros(batch_dim, num_experts, in_dim))
        self.norm_scale = nn.Parameter(torch.ones(batch_dim, in_dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        up_gate = torch.einsum("dbi,deih->dbeh", x, self.w_up) + self.b_up.unsqueeze(1)
        up, gate = up_gate.chunk(2, -1)
        hidden = F.silu(gate) * up
        outs = torch.einsum("dbeh,dehi->dbei", hidden, self.w_down) + self.b_down.unsqueeze(1)
        if self.num_experts == 1:
            moe = outs[:, :, 0]
        else:
            logits = torch.einsum("dbi,dio->dbo", x, self.w_gate) + self.b_gate.unsqueeze(1)
            if self.sparse:
                val, idx = logits.topk(self.top_k, -1)
                w = fp32_softmax(val, -1)
                picked = torch.gather(outs, 2, idx.unsqueeze(-1).expand(*idx.shape, self.in_dim))
                moe = (picked * w.unsqueeze(-1)).sum(2)
            else:
                moe = (outs * fp32_softmax(logits, -1).unsqueeze(-1)).sum(2)
        if self.residual_norm:
            return fp32_rms_normalize(x + moe, -1) * self.norm_scale.unsqueeze(1)
        return moe


class RMSNorm(nn.Module):
    """RMS normalisation over the last dim in fp32 with a learnable scale (eps 1e-6)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return (fp32_rms_normalize(x, -1, self.eps) * self.scale.float()).to(x.dtype)


def _head_major(x: torch.Tensor, heads: int) -> torch.Tensor:
    """[B, T, D] -> [heads, B, T * D / heads]: every head sees its slice of every token."""
    B, T, D = x.shape
    return x.reshape(B, T, heads, D // heads).permute(2, 0, 1, 3).reshape(heads, B, T * (D // heads))


def _token_major(y: torch.Tensor, tokens: int) -> torch.Tensor:
    """[heads, B, T * hd] -> [T, B, heads * hd]: back to one row per token (heads concatenated)."""
    H, B, _ = y.shape
    return y.reshape(H, B, tokens, -1).permute(2, 1, 0, 3).reshape(tokens, B, -1)


class TokenMixLargeMoe(nn.Module):
    """Multi-head token mixing with MoE feed-forwards, mean-pooled over tokens.

    Each of ``layer_num`` layers runs a ``BatchedExpertMoE`` over heads (one expert bank per head,
    input = that head's slice of all tokens) and then one over tokens (one bank per token, input =
    the token's heads concatenated).  Input [B, token_num, token_dim]; output [B, token_dim].
    Reference behaviour: src/flare/jax/layers/token_mix.py:147-223.
    """

    def __init__(self, layer_num: int, token_num: int, token_dim: int, head_num: int = 12, scale_size: int = 4,
                 num_experts: int = 1, sparse: bool = False, top_k: int = 2):
        super().__init__()
        if token_dim % head_num:
            raise ValueError(f"token_dim {token_dim} must be divisible by head_num {head_num}")
        self.layer_num, self.token_num, self.token_dim, self.head_num = layer_num, token_num, token_dim, head_num
        self.head_dim = token_dim // head_num
        k = min(top_k, num_experts)
        self.head_moe = nn.ModuleList(BatchedExpertMoE(head_num, token_num * self.head_dim, scale_size, num_experts,
                                                       sparse, k) for _ in range(layer_num))
        self.token_moe = nn.ModuleList(BatchedExpertMoE(token_num, token_dim, scale_size, num_experts, sparse, k)
                                       for _ in range(layer_num))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for i in range(self.layer_num):
            y = self.head_moe[i](_head_major(x, self.head_num))
            x = self.token_moe[i](_token_major(y, self.token_num)).transpose(0, 1)
        return fp32_mean(x, dim=1)


class TokenMixLargePreGateNoPool(nn.Module):
    """``TokenMixLargeMoe`` with per-layer input gates, pre-norm residual MoE blocks and no pooling.

    ``forward(x, pre_layer_gates)``: before layer i the tokens are scaled by
    ``pre_layer_gates[:, i*D:(i+1)*D]`` (one gate vector per sample, shared by the tokens); each MoE
    block is ``y = y + MoE(RMSNorm(y))``; layers listed in ``residual_layers`` (with
    ``residual_enabled``) also normalise their input and add it back after the layer.  Output
    [B, token_num, token_dim].  Reference behaviour: src/flare/jax/layers/token_mix.py:226-335.
    """

    def __init__(self, layer_num: int, token_num: int, token_dim: int, head_num: int = 12, scale_size: int = 4,
                 num_experts: int = 1, sparse: bool = False, top_k: int = 2, residual_enabled: bool = False,
                 residual_layers: Sequence[int] = ()):
        super().__init__()
        if token_dim % head_num:
            raise ValueError(f"token_dim {token_dim} must be divisible by head_num {head_num}")
        for li in residual_layers:
            if not 0 <= li < layer_num:
                raise ValueError(f"residual layer index {li} is outside [0, {layer_num})")
        self.layer_num, self.token_num, self.token_dim, self.head_num = layer_num, token_num, token_dim, head_num
        self.head_dim = token_dim // head_num
        self.residual_enabled, self.residual_layers = residual_enabled, frozenset(residual_layers)
        k = min(top_k, num_experts)
        hw = token_num * self.head_dim
        self.head_moe = nn.ModuleList(BatchedExpertMoE(head_num, hw, scale_size, num_experts, sparse, k,
                                                       residual_norm=False) for _ in range(layer_num))
        self.token_moe = nn.ModuleList(BatchedExpertMoE(token_num, token_dim, scale_size, num_experts, sparse, k,
                                                        residual_norm=False) for _ in range(layer_num))
        self.head_norms = nn.ModuleList(RMSNorm(hw) for _ in range(layer_num))
        self.token_norms = nn.ModuleList(RMSNorm(token_dim) for _ in range(layer_num))
        self.block_norms = nn.ModuleDict({str(i): RMSNorm(token_dim) for i in sorted(self.residual_layers)})

    def forward(self, x: torch.Tensor, pre_layer_gates: torch.Tensor | None = None) -> torch.Tensor:
        D = self.token_dim
        for i in range(self.layer_num):
            if pre_layer_gates is not None:
                x = x * pre_layer_gates[:, i * D:(i + 1) * D].unsqueeze(1)
            block_in = x
            res = self.residual_enabled and i in self.residual_layers
            if res:
                x = self.block_norms[str(i)](x)
            y = _head_major(x, self.head_num)
            y = y + self.head_moe[i](self.head_norms[i](y))
            t = _token_major(y, self.token_num)
            t = t + self.token_moe[i](self.token_norms[i](t))
            x = t.transpose(0, 1)
            if res:
                x = x + block_in
        return x


class NamedTokens:
    """Ordered name -> token index registry for token-mixing models."""

    def __init__(self, names: Sequence[str]):
        if len(set(names)) != len(names):
            raise ValueError("token names must be unique")
        self.names = tuple(names)
        self.index = {n: i for i, n in enumerate(self.names)}

    def __len__(self) -> int:
        return len(self.names)

    def select(self, tokens: torch.Tensor, names: Sequence[str]) -> torch.Tensor:
        return tokens[:, [self.index[n] for n in names]]


__all__ = ["BatchedExpertMoE", "CGC", "CategoricalEmbedding", "MLP", "NamedTokens", "PLE", "RMSNorm", "TcLinear",
           "TokenMix", "TokenMixLargeMoe", "TokenMixLargePreGateNoPool", "UCGC", "UPLE", "fp32_mean",
           "fp32_rms_normalize", "fp32_softmax", "fp32_sum", "get_activation"]
