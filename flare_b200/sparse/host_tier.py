"""Host-DRAM tier for embedding tables larger than HBM.

A table spec with ``cache_rows`` set keeps every row (and its optimizer state)
in pinned host memory; the collection holds ``cache_rows`` HBM slots for it and
a device row -> slot map that the fused forward reads (ids of non-resident
rows are an error: placement always happens before the step).

``HostTier`` runs the placement one step ahead, on the host, because the host
holds the next batch's ids before the GPU needs them:

1. ``plan(t, ids)``: mark the step's resident rows as used at step ``t``, pick
   victim slots for the misses with a CLOCK sweep over slots not used by
   steps ``t-1`` (possibly still running) or ``t``, and update the host-side
   directory;
2. ``issue(plan)`` on a side stream: gather the victims' rows + state from
   their slots into a device staging buffer and copy them to pinned host
   memory (write-back, scattered into the host arrays before the next plan
   gathers), gather the missed rows from the host arrays into pinned staging
   and copy them with ONE ``cudaMemcpyAsync`` per array, then one kernel maps
   the rows to their slots and scatters them in;
3. the training step's stream waits for the plan's event, then runs the fused
   kernels unchanged (their ids go through the row -> slot map).

The plan for step ``t+1`` can be issued while step ``t`` runs: its victims are
never slots step ``t`` uses.  With several ranks each owner needs the ids of
every rank's batch for the tables it owns; they are all-gathered on a gloo
group on the host.  The reference's larger-than-RAM tier is a host-memory
limit with disk spill inside its external store
(src/flare/runtime/fluxway/workers/sparse_storage.py); its primary copy is
host memory and it has no HBM cache.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .._native import native
from ..ops.dense import init_uniform_


@dataclass
class ShardPlan:
    step: int
    miss_rows: np.ndarray    # int64 rows fetched from host
    miss_slots: np.ndarray   # int32 their slots
    evict_rows: np.ndarray   # int64 rows written back (evicted)
    evict_slots: np.ndarray  # int32 their slots
    hits: int


class HostShard:
    """Host copy + directory of one host-tier shard of a collection."""

    STAGE_ROWS0 = 1 << 16

    def __init__(self, coll, i: int, seed: int):
        s = coll.shards[i]
        self.coll, self.i, self.shard = coll, i, s
        self.rows, self.ncols, self.C = s.spec.num_embeddings, s.ncols, s.storage_rows
        dev = coll.device
        self.w = torch.empty(self.rows, self.ncols, dtype=torch.float32, pin_memory=True)
        # same counter-based init as a resident table: generate on the device in chunks, copy to host
        stream_seed = (seed * 1_000_003 + s.table * 7919) & 0x7FFFFFFF
        chunk = max(1, (1 << 26) // self.ncols)
        buf = torch.empty(chunk * self.ncols, dtype=torch.float32, device=dev)
        for r0 in range(0, self.rows, chunk):
            n = min(chunk, self.rows - r0)
            init_uniform_(buf[:n * self.ncols], -s.spec.init_scale, s.spec.init_scale, stream_seed,
                          index_offset=r0 * s.spec.embedding_dim, ncols=self.ncols, dim=s.spec.embedding_dim,
                          col_begin=s.col_begin)
            self.w[r0:r0 + n].copy_(buf[:n * self.ncols].view(n, self.ncols))
        del buf
        f = coll.shard_fields(i)
        self.cache_w = f["weight"]
        self.cache_row = f.get("state_row")
        self.cache_m, self.cache_v = f.get("state_m"), f.get("state_v")
        pin = dict(dtype=torch.float32, pin_memory=True)
        self.h_row = torch.zeros(self.rows, **pin) if self.cache_row is not None else None
        self.h_m = torch.zeros(self.rows, self.ncols, **pin) if self.cache_m is not None else None
        self.h_v = torch.zeros(self.rows, self.ncols, **pin) if self.cache_v is not None else None
        self.slot_map = coll.slot_map[s.slot_map_off:s.slot_map_off + self.rows]
        self.slot_of = np.full(self.rows, -1, dtype=np.int32)
        self.row_of = np.full(self.C, -1, dtype=np.int64)
        self.stamp = np.full(self.C, -(1 << 40), dtype=np.int64)
        self.hand = 0
        self._stage_cap = 0
        self._pending_wb: tuple | None = None
        self._h2d_done: torch.cuda.Event | None = None  # the pinned fetch staging is free once this fires
        self.stats = {"hits": 0, "misses": 0, "evictions": 0}

    # ------------------------------------------------------------ staging
    def _ensure_stage(self, n: int) -> None:
        if n <= self._stage_cap:
            return
        cap = max(n, self.STAGE_ROWS0, 2 * self._stage_cap)
        dev = self.coll.device
        mk_h = lambda *shape: torch.empty(*shape, dtype=torch.float32, pin_memory=True)  # noqa: E731
        mk_d = lambda *shape: torch.empty(*shape, dtype=torch.float32, device=dev)  # noqa: E731
        self.hs = {"w": mk_h(cap, self.ncols)}  # fetch staging (host)
        self.ds = {"w": mk_d(cap, self.ncols)}  # fetch staging (device)
        self.hwb = {"w": mk_h(cap, self.ncols)}  # write-back staging (host)
        self.dwb = {"w": mk_d(cap, self.ncols)}  # write-back staging (device)
        for name, cache, width in (("row", self.cache_row, None), ("m", self.cache_m, self.ncols),
                                   ("v", self.cache_v, self.ncols)):
            if cache is None:
                continue
            shape = (cap,) if width is None else (cap, width)
            self.hs[name], self.ds[name] = mk_h(*shape), mk_d(*shape)
            self.hwb[name], self.dwb[name] = mk_h(*shape), mk_d(*shape)
        self.d_rows = torch.empty(cap, dtype=torch.int64, device=dev)
        self.d_evict = torch.empty(cap, dtype=torch.int64, device=dev)
        self.d_slots = torch.empty(cap, dtype=torch.int32, device=dev)
        self.d_wslots = torch.empty(cap, dtype=torch.int32, device=dev)
        self.h_idx = torch.empty(cap, dtype=torch.int64, pin_memory=True)
        self.h_idx2 = torch.empty(cap, dtype=torch.int64, pin_memory=True)
        self.h_slots = torch.empty(cap, dtype=torch.int32, pin_memory=True)
        self.h_wslots = torch.empty(cap, dtype=torch.int32, pin_memory=True)
        self._stage_cap = cap

    # --------------------------------------------------------------- plan
    def _claim(self, n: int, step: int) -> np.ndarray:
        """n victim slots not used by steps step-1 or step (CLOCK sweep from the hand)."""
        out = []
        need, C = n, self.C
        scanned = 0
        while need > 0:
            if scanned >= C:
                raise RuntimeError(f"host-tier cache of {C} rows cannot hold two consecutive steps' rows")
            w = min(C - self.hand, max(4 * need, 1 << 16))
            cand = np.nonzero(self.stamp[self.hand:self.hand + w] < step - 1)[0] + self.hand
            take = cand[:need]
            self.stamp[take] = step  # claimed: never handed out twice
            out.append(take)
            need -= len(take)
            if need == 0 and len(take):
                self.hand = int(take[-1] + 1) % C
            else:
                self.hand = (self.hand + w) % C
            scanned += w
        return np.concatenate(out).astype(np.int32) if out else np.zeros(0, np.int32)

    def plan(self, step: int, rows: np.ndarray) -> ShardPlan:
        rows = np.unique(rows.astype(np.int64))
        if len(rows) and (rows[0] < 0 or rows[-1] >= self.rows):
            raise ValueError("ids outside the table")
        slots = self.slot_of[rows]
        res = slots >= 0
        self.stamp[slots[res]] = step
        miss = rows[~res]
        if len(miss) > self.C:
            raise RuntimeError("one step touches more rows than the host-tier cache holds")
        vs = self._claim(len(miss), step)
        vrows = self.row_of[vs]
        ev = vrows >= 0
        evict_rows, evict_slots = vrows[ev], vs[ev]
        self.slot_of[evict_rows] = -1
        self.slot_of[miss] = vs
        self.row_of[vs] = miss
        self.stamp[vs] = step
        self.stats["hits"] += int(res.sum())
        self.stats["misses"] += len(miss)
        self.stats["evictions"] += len(evict_rows)
        return ShardPlan(step, miss, vs, evict_rows, evict_slots, int(res.sum()))

    # -------------------------------------------------------------- issue
    def finish_writeback(self) -> None:
        """Scatter the previous plan's written-back rows into the host arrays (waits for its copy)."""
        if self._pending_wb is None:
            return
        ev, rows, n = self._pending_wb
        ev.synchronize()
        idx = torch.from_numpy(rows)
        self.w.index_copy_(0, idx, self.hwb["w"][:n])
        if self.h_row is not None:
            self.h_row.index_copy_(0, idx, self.hwb["row"][:n])
        if self.h_m is not None:
            self.h_m.index_copy_(0, idx, self.hwb["m"][:n])
        if self.h_v is not None:
            self.h_v.index_copy_(0, idx, self.hwb["v"][:n])
        self._pending_wb = None

    def issue(self, p: ShardPlan, stream: torch.cuda.Stream) -> None:
        """Enqueue write-back and fetch of plan ``p`` on ``stream`` (host gathers happen now)."""
        C = native()
        self.finish_writeback()
        if self._h2d_done is not None:  # the previous plan's copies still read the pinned staging
            self._h2d_done.synchronize()
            self._h2d_done = None
        n, ne = len(p.miss_rows), len(p.evict_rows)
        self._ensure_stage(max(n, ne, 1))
        # host gather of the missed rows (the write-back of any of them finished above)
        if n:
            idx = torch.from_numpy(p.miss_rows)
            torch.index_select(self.w, 0, idx, out=self.hs["w"][:n])
            if self.h_row is not None:
                torch.index_select(self.h_row, 0, idx, out=self.hs["row"][:n])
            if self.h_m is not None:
                torch.index_select(self.h_m, 0, idx, out=self.hs["m"][:n])
            if self.h_v is not None:
                torch.index_select(self.h_v, 0, idx, out=self.hs["v"][:n])
            self.h_idx[:n].copy_(idx)
            self.h_slots[:n].copy_(torch.from_numpy(p.miss_slots))
        if ne:
            self.h_idx2[:ne].copy_(torch.from_numpy(p.evict_rows))
            self.h_wslots[:ne].copy_(torch.from_numpy(p.evict_slots))
        with torch.cuda.stream(stream):
            if ne:
                self.d_wslots[:ne].copy_(self.h_wslots[:ne], non_blocking=True)
                C.tier_gather(self._params(ne, self.d_wslots, self.dwb))
                for k in self.dwb:
                    self.hwb[k][:ne].copy_(self.dwb[k][:ne], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
                self._pending_wb = (ev, p.evict_rows.copy(), ne)
                self.d_evict[:ne].copy_(self.h_idx2[:ne], non_blocking=True)
            if n:
                for k in self.hs:
                    self.ds[k][:n].copy_(self.hs[k][:n], non_blocking=True)
                self.d_rows[:n].copy_(self.h_idx[:n], non_blocking=True)
                self.d_slots[:n].copy_(self.h_slots[:n], non_blocking=True)
            if n or ne:
                self._h2d_done = torch.cuda.Event()
                self._h2d_done.record(stream)
            if n or ne:
                d = self._params(n, self.d_slots, self.ds)
                d.update(slot_map=self.slot_map.data_ptr(), new_rows=self.d_rows.data_ptr(),
                         evict_rows=self.d_evict.data_ptr(), n_evict=ne)
                C.tier_install(d)

    def _params(self, n: int, slots: torch.Tensor, stage: dict) -> dict:
        d = {"n": n, "ncols": self.ncols, "slots": slots.data_ptr(), "cache_w": self.cache_w.data_ptr(),
             "stage_w": stage["w"].data_ptr()}
        for name, cache in (("row", self.cache_row), ("m", self.cache_m), ("v", self.cache_v)):
            if cache is not None:
                d["cache_" + name] = cache.data_ptr()
                d["stage_" + name] = stage[name].data_ptr()
        return d

    # ------------------------------------------------------------- export
    def flush(self) -> None:
        """Write every resident row back to the host arrays (synchronous)."""
        self.finish_writeback()
        res = np.nonzero(self.row_of >= 0)[0].astype(np.int32)
        if len(res) == 0:
            return
        rows = self.row_of[res]
        slots = torch.from_numpy(res).to(self.coll.device)
        idx = torch.from_numpy(rows)
        self.w.index_copy_(0, idx, self.cache_w.index_select(0, slots.long()).cpu())
        if self.h_row is not None:
            self.h_row.index_copy_(0, idx, self.cache_row.index_select(0, slots.long()).cpu())
        if self.h_m is not None:
            self.h_m.index_copy_(0, idx, self.cache_m.index_select(0, slots.long()).cpu())
        if self.h_v is not None:
            self.h_v.index_copy_(0, idx, self.cache_v.index_select(0, slots.long()).cpu())


class HostTier:
    """Placement driver for every host-tier shard this rank owns."""

    def __init__(self, coll, *, seed: int = 0):
        self.coll = coll
        self.shards = [HostShard(coll, i, seed) for i, s in enumerate(coll.shards) if s.slot_map_off >= 0]
        self.stream = torch.cuda.Stream(device=coll.device)
        self.ready = torch.cuda.Event()
        self._group = None
        if coll.world > 1:
            import torch.distributed as dist

            self._group = dist.new_group(backend="gloo")
        self.features = coll.features

    def _owned_ids(self, offsets: torch.Tensor, values: torch.Tensor) -> dict[int, np.ndarray]:
        """ids of every rank's batch for the features of this rank's host-tier shards."""
        B, F = self.coll.B, self.coll.F
        off = offsets.cpu().numpy() if offsets.is_cuda else offsets.numpy()
        vals = values.cpu().numpy() if values.is_cuda else values.numpy()
        per_feature = {f: vals[off[f * B]:off[(f + 1) * B]] for f in range(F)}
        if self._group is None:
            return per_feature
        import torch.distributed as dist

        parts = [None] * self.coll.world
        dist.all_gather_object(parts, per_feature, group=self._group)
        return {f: np.concatenate([p[f] for p in parts]) for f in range(F)}

    def prepare(self, step: int, offsets: torch.Tensor, values: torch.Tensor,
                wait_for: torch.cuda.Event | None = None) -> torch.cuda.Event:
        """Make every row of step ``step``'s batch resident; returns the event the step must wait for."""
        ids = self._owned_ids(offsets, values)
        if wait_for is not None:
            self.stream.wait_event(wait_for)
        for hs in self.shards:
            f = self.features.index(hs.shard.spec.feature_name)
            hs.issue(hs.plan(step, ids[f]), self.stream)
        self.ready.record(self.stream)
        return self.ready

    def stats(self) -> dict:
        out = {"hits": 0, "misses": 0, "evictions": 0}
        for hs in self.shards:
            for k in out:
                out[k] += hs.stats[k]
        return out

    def flush(self) -> None:
        torch.cuda.synchronize(self.coll.device)
        for hs in self.shards:
            hs.flush()

    def host_bytes(self) -> int:
        tot = 0
        for hs in self.shards:
            for t in (hs.w, hs.h_row, hs.h_m, hs.h_v):
                if t is not None:
                    tot += t.numel() * t.element_size()
        return tot


__all__ = ["HostShard", "HostTier", "ShardPlan"]
