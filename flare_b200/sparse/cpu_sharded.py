"""Table-wise sharded CPU embedding collection over torch.distributed (gloo) ranks.

The host counterpart of the fused GPU exchange: table f lives on rank
``f % world``; every rank holds the keyed-jagged batch of its own samples.

* forward: each rank sends, to every owner, the bag lengths and ids of the
  owner's tables for its ``B`` samples (two ``all_to_all_single`` calls);
  the owner pools the global batch of its tables (samples in rank order)
  with an ordinary ``CpuEmbeddingBagCollection`` and sends every rank the
  pooled rows of its samples (a third ``all_to_all_single``); each rank
  assembles ``[B, total_dim]`` in table order.
* backward: each rank sends the owners the pooled gradients of their tables
  (one ``all_to_all_single``); the owner applies the row-wise optimizer once
  for the whole global batch.

With gradients that follow the sample-mean contract (each rank's divided by
the world size, ``TrainEngine.input_gradients``) the tables evolve exactly as
one collection trained on the concatenated batch.  Reference behaviour: the
routed lookup / update of the sparse tables (src/flare/runtime/fluxway/
workers/sparse_input.py:447-455, dynamic_embedding.py:362-397, 551-560),
which the reference runs on Ray workers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .config import SparseOptimizerConfig, SparseTableSpec
from .reference import CpuEmbeddingBagCollection


class ShardedCpuEmbeddingBagCollection:
    def __init__(self, tables: list[SparseTableSpec], batch_size: int, *, optimizer: SparseOptimizerConfig | None = None,
                 seed: int = 0, native: bool = True, group=None, weights: list[torch.Tensor] | None = None):
        self.tables, self.B, self.group = list(tables), int(batch_size), group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.F = len(tables)
        self.owner = [f % self.world for f in range(self.F)]
        self.owned = [f for f in range(self.F) if self.owner[f] == self.rank]
        self.by_owner = [[f for f in range(self.F) if self.owner[f] == r] for r in range(self.world)]
        self.dims = [t.embedding_dim for t in tables]
        self.col = [sum(self.dims[:f]) for f in range(self.F)]
        self.total_dim = sum(self.dims)
        opt = optimizer or tables[0].optimizer
        self.local = None
        if self.owned:
            # table f's initial rows depend only on (seed, f), whatever the rank that owns it
            init = weights if weights is not None else [None] * self.F
            w = [init[f] if init[f] is not None else
                 CpuEmbeddingBagCollection([tables[f]], 1, optimizer=opt, seed=seed * 1_000_003 + f).weights[0]
                 for f in self.owned]
            self.local = CpuEmbeddingBagCollection([tables[f] for f in self.owned], self.world * self.B, optimizer=opt,
                                                   weights=w, native=native, seed=seed)

    def _a2a(self, send: list[torch.Tensor], recv_sizes: list[int], dtype) -> list[torch.Tensor]:
        out = torch.empty(sum(recv_sizes), dtype=dtype)
        inp = torch.cat([s.reshape(-1).to(dtype) for s in send]) if send else torch.empty(0, dtype=dtype)
        if self.world > 1:
            dist.all_to_all_single(out, inp, recv_sizes, [s.numel() for s in send], group=self.group)
        else:
            out.copy_(inp)
        return list(torch.split(out, recv_sizes))

    def set_input(self, offsets: torch.Tensor, values: torch.Tensor, non_blocking: bool = False) -> None:
        B, W = self.B, self.world
        offs, vals = offsets.cpu().long(), values.cpu()
        lens = offs[1:] - offs[:-1]
        send_len, send_val = [], []
        for r in range(W):
            fs = self.by_owner[r]
            send_len.append(torch.cat([lens[f * B:(f + 1) * B] for f in fs]) if fs else torch.empty(0, dtype=torch.long))
            send_val.append(torch.cat([vals[int(offs[f * B]):int(offs[(f + 1) * B])] for f in fs]) if fs
                            else torch.empty(0, dtype=vals.dtype))
        mine = len(self.owned) * B
        rlens = self._a2a(send_len, [mine] * W, torch.int64)
        counts = self._a2a([torch.tensor([v.numel()]) for v in send_val], [1] * W, torch.int64)
        rvals = self._a2a(send_val, [int(c) for c in counts], torch.int32)
        if not self.owned:
            return
        # the owner's global batch: table-major, then source rank, then sample
        n_own = len(self.owned)
        per_src = [rl.reshape(n_own, B) for rl in rlens]
        val_src = []
        for s in range(W):
            cut = torch.cumsum(per_src[s].sum(1), 0)
            starts = torch.cat([torch.zeros(1, dtype=torch.long), cut[:-1]])
            val_src.append([rvals[s][int(a):int(a + n)] for a, n in zip(starts, per_src[s].sum(1))])
        g_lens = torch.cat([torch.cat([per_src[s][k] for s in range(W)]) for k in range(n_own)])
        g_vals = torch.cat([torch.cat([val_src[s][k] for s in range(W)]) for k in range(n_own)])
        g_offs = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(g_lens, 0)]).int()
        self.local.set_input(g_offs, g_vals.int())

    def forward(self, training: bool = True) -> torch.Tensor:
        B, W = self.B, self.world
        send = []
        if self.owned:
            pooled = self.local.forward(training)  # [W*B, own_dim]
            send = [pooled[s * B:(s + 1) * B] for s in range(W)]
        else:
            send = [torch.empty(0) for _ in range(W)]
        recv = self._a2a(send, [B * sum(self.dims[f] for f in self.by_owner[r]) for r in range(W)], torch.float32)
        out = torch.zeros(B, self.total_dim)
        for r in range(W):
            fs = self.by_owner[r]
            if not fs:
                continue
            block = recv[r].reshape(B, -1)
            c = 0
            for f in fs:
                out[:, self.col[f]:self.col[f] + self.dims[f]] = block[:, c:c + self.dims[f]]
                c += self.dims[f]
        return out

    def backward(self, grad_pooled: torch.Tensor, step: int | None = None) -> None:
        B, W = self.B, self.world
        g = grad_pooled.detach().float()
        send = [torch.cat([g[:, self.col[f]:self.col[f] + self.dims[f]] for f in self.by_owner[r]], 1)
                if self.by_owner[r] else torch.empty(0) for r in range(W)]
        own_dim = sum(self.dims[f] for f in self.owned)
        recv = self._a2a(send, [B * own_dim] * W, torch.float32)
        if self.owned:
            self.local.backward(torch.cat([x.reshape(B, own_dim) for x in recv]), step)

    def state_dict(self) -> dict:
        """This rank's owned tables (whole, by name), their optimizer state and dynamic key maps."""
        st = self.local.state_dict() if self.local is not None else {"tables": {}, "dynamic": {}, "step": 0}
        return {**st, "world": self.world, "rank": self.rank}

    def load_state_dict(self, states) -> None:
        """Restore from one state or from every rank's states of a run at any world size (tables are
        whole per owner, so the union of the states holds every table)."""
        states = [states] if isinstance(states, dict) else list(states)
        if self.local is None:
            return
        # every table's entry carries its own row-init stream, so the union restores each table exactly
        merged = {"tables": {}, "dynamic": {}, "step": max(int(s.get("step", 0)) for s in states)}
        for s in states:
            merged["tables"].update(s["tables"])
            merged["dynamic"].update(s.get("dynamic", {}))
            if "optimizer" in s:
                merged["optimizer"] = s["optimizer"]
        self.local.load_state_dict(merged)

    def table_weights(self, f: int) -> torch.Tensor | None:
        """Table f's weights on its owner (None elsewhere)."""
        return self.local.table_weights(self.owned.index(f)) if f in self.owned else None


def slice_samples(offsets: torch.Tensor, values: torch.Tensor, num_features: int, batch: int, lo: int,
                  hi: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Samples [lo, hi) of a feature-major keyed-jagged batch of ``batch`` samples (a rank's share)."""
    offs = offsets.long()
    lens, vals = [], []
    for f in range(num_features):
        a, b = f * batch + lo, f * batch + hi
        lens.append(offs[a + 1:b + 1] - offs[a:b])
        vals.append(values[int(offs[a]):int(offs[b])])
    ls = torch.cat(lens)
    return torch.cat([torch.zeros(1, dtype=torch.long), ls.cumsum(0)]).to(offsets.dtype), torch.cat(vals)


__all__ = ["ShardedCpuEmbeddingBagCollection", "slice_samples"]
