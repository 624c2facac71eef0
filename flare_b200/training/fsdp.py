"""FSDP (ZeRO-3) weights whose all-gather is fused into the consuming GEMM.

A ``FsdpWeight`` is a 2-D weight ``[rows, cols]`` split into row blocks over a
group of ranks.  Every member keeps:

* the fp32 master rows, Adam moments and nothing else of its block
  (ZeRO-3 ownership, src/flare/training/zero/contracts.py:58-62);
* a bf16 compute copy in a ``ShardedRows`` buffer: the member writes its own
  rows after each update; the first GEMM that reads the weight pulls the
  other members' rows over NVLink inside the GEMM kernel
  (ops/dist_gemm.py), and later GEMMs of the same step read the local copy;
* an fp32 gradient of the whole matrix in symmetric memory (weight-gradient
  GEMMs accumulate into it).

``apply()`` runs one kernel that reduce-scatters the gradient over the group
(each member sums the peers' rows of its block over NVLink and zeroes them),
applies Adam/AdamW to its block and writes the bf16 rows of its block.  The
parameter all-gather of the next step happens inside the next forward GEMM.
The reference gathers ZeRO-3 parameters with separate XLA all-gathers per
micro-step (src/flare/jax/training/state/layout.py:176-194) and reduce-
scatters gradients with ``psum_scatter`` (src/flare/jax/training/zero/
collectives.py:38-40).
"""
from __future__ import annotations

import torch

from .._native import native
from ..ops.dist_gemm import DistGemmContext, ShardedRows
from ..parallel.symm import FlagRegion
from .flat import DenseOptimizerConfig, adam_reference


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class FsdpGroup:
    """Barrier flags + epoch words shared by every FSDP weight of one rank group."""

    def __init__(self, ctx: DistGemmContext, group: list[int]):
        self.ctx, self.group = ctx, list(group)
        self.R = len(group)
        self.my = self.group.index(ctx.rank)
        self.flags = FlagRegion(ctx.heap, 2)
        dev = ctx.device
        self.peer_flags = torch.tensor([self.flags.buf.peer_ptrs[g] for g in self.group], dtype=torch.int64,
                                       device=dev)


class FsdpWeight:
    def __init__(self, fg: FsdpGroup, name: str, rows: int, cols: int, *, init_scale: float, seed: int,
                 opt: DenseOptimizerConfig, step_dev: torch.Tensor, row_multiple: int = 64,
                 full_init: torch.Tensor | None = None):
        self.fg, self.name, self.opt = fg, name, opt
        ctx = fg.ctx
        R = fg.R
        self.rows, self.cols = int(rows), int(cols)
        self.ld = _round_up(cols, 8)
        S = _round_up(-(-self.rows // R), row_multiple)
        self.S = S
        self.w = ShardedRows(ctx, fg.group, S, self.cols, ld=self.ld)
        self.grad_buf = ctx.heap.alloc((R * S, self.ld), torch.float32)
        self.grad_buf.local.zero_()
        self.peer_grad = torch.tensor([self.grad_buf.peer_ptrs[g] for g in fg.group], dtype=torch.int64,
                                      device=ctx.device)
        self.peer_param = torch.tensor([self.w.buf.local.data_ptr()], dtype=torch.int64, device=ctx.device)
        # deterministic init of the whole matrix, this member keeps its block
        if full_init is None:
            g = torch.Generator().manual_seed(seed)
            full_init = torch.randn(self.rows, self.cols, generator=g) * init_scale
        full = torch.zeros(R * S, self.ld)
        full[:self.rows, :self.cols] = full_init
        lo = fg.my * S
        self.master = full[lo:lo + S].reshape(-1).to(ctx.device).contiguous()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.w.local.copy_(full[lo:lo + S].to(torch.bfloat16))
        self.step_dev = step_dev
        self.status = ctx.status

    # ------------------------------------------------------------------ views
    @property
    def full(self) -> torch.Tensor:
        """bf16 [rows, cols] compute copy (complete after a gathering GEMM this step)."""
        return self.w.full[:self.rows, :self.cols]

    @property
    def grad(self) -> torch.Tensor:
        """fp32 [rows, cols] local gradient accumulator."""
        return self.grad_buf.local[:self.rows, :self.cols]

    def numel(self) -> int:
        return self.rows * self.cols

    # -------------------------------------------------------------- optimizer
    def apply(self, step: int, grad_scale: float = 1.0) -> None:
        op = self.opt.kernel_params(step)
        op["step_ptr"] = self.step_dev.data_ptr()
        fg = self.fg
        n_shard = self.S * self.ld
        native().adam_dp_fused(dict(
            world=fg.R, rank=fg.my, lo=fg.my * n_shard, hi=(fg.my + 1) * n_shard,
            peer_grad=self.peer_grad.data_ptr(), peer_param=self.peer_param.data_ptr(), param_world=1,
            master_shard=self.master.data_ptr(), m_shard=self.m.data_ptr(), v_shard=self.v.data_ptr(),
            grad_scale=float(grad_scale), opt=op, flags_local=fg.flags.local_ptr,
            peer_flags=fg.peer_flags.data_ptr(), flag_in=fg.flags.slots(0), flag_out=fg.flags.slots(1),
            epoch_ctr=fg.flags.epoch_ptr(0), block_counter=fg.flags.block_counter_ptr(0), status=self.status.ptr,
            timeout_ns=fg.ctx.timeout_ns))

    def master_rows(self) -> torch.Tensor:
        """This member's fp32 block [S, cols]."""
        return self.master.view(self.S, self.ld)[:, :self.cols]

    def gather_master(self) -> torch.Tensor:
        """Full fp32 [rows, cols] (collective over the group when R > 1; gloo/nccl all_gather)."""
        if self.fg.R == 1:
            return self.master_rows()[:self.rows].clone()
        import torch.distributed as dist

        parts = [torch.empty(self.S * self.ld, device=self.master.device) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, self.master)
        rows = [parts[g].view(self.S, self.ld)[:, :self.cols] for g in self.fg.group]
        return torch.cat(rows)[:self.rows]


__all__ = ["FsdpGroup", "FsdpWeight", "adam_reference"]
