"""Host-DRAM tier for embedding tables larger than HBM (device-driven placement).

A table spec with ``cache_rows`` set keeps every row (and its optimizer state)
in pinned host memory; the collection holds ``cache_rows`` HBM slots for it and
a device row -> slot map that the fused forward reads.  ``HostTier.prepare``
(called by the collection at the start of every forward) launches two kernels
(``csrc/host_tier.cu``) that make every row of the step resident: hits stamp
their slots, each missing row claims a victim slot with a device CLOCK sweep,
the victim is written back to host memory and the row pulled from it, both
directly over PCIe through the pinned memory's device address.  The host does
nothing per step, so the step (placement included) replays from one CUDA
graph, and the PCIe traffic overlaps whatever else the GPU runs.

The reference's larger-than-RAM tier is a memory limit with disk spill inside
its external store (src/flare/runtime/fluxway/workers/sparse_storage.py); its
primary copy is host memory and it keeps no HBM cache.
"""
from __future__ import annotations

import torch

from .._native import native
from ..ops.dense import init_uniform_

INT_MIN = -(1 << 31)


class HostShard:
    """Host copy + device directory of one host-tier shard of a collection."""

    def __init__(self, coll, i: int, seed: int):
        s = coll.shards[i]
        self.coll, self.i, self.shard = coll, i, s
        self.rows, self.ncols, self.C = s.spec.num_embeddings, s.ncols, s.storage_rows
        dev = coll.device
        self.w = torch.empty(self.rows, self.ncols, dtype=torch.float32, pin_memory=True)
        # the same counter-based init as a resident table: generate on the device in chunks, copy to host
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
        self.slot2row = torch.full((self.C,), -1, dtype=torch.int64, device=dev)
        self.stamp = torch.full((self.C,), INT_MIN, dtype=torch.int32, device=dev)
        self.hand = torch.zeros(1, dtype=torch.int32, device=dev)
        self.miss_cap = coll.world * coll.stage_cap
        self.miss_rows = torch.empty(self.miss_cap, dtype=torch.int32, device=dev)
        self.num_miss = torch.zeros(1, dtype=torch.int32, device=dev)

    def params(self) -> dict:
        d = {"feature": self.coll.features.index(self.shard.spec.feature_name), "ncols": self.ncols,
             "rows": self.rows, "C": self.C, "slot_map": self.slot_map.data_ptr(),
             "slot2row": self.slot2row.data_ptr(), "stamp": self.stamp.data_ptr(), "hand": self.hand.data_ptr(),
             "cache_w": self.cache_w.data_ptr(), "host_w": self.w.data_ptr(),
             "miss_rows": self.miss_rows.data_ptr(), "num_miss": self.num_miss.data_ptr(),
             "miss_cap": self.miss_cap}
        for name, cache, host in (("row", self.cache_row, self.h_row), ("m", self.cache_m, self.h_m),
                                  ("v", self.cache_v, self.h_v)):
            if cache is not None:
                d["cache_" + name] = cache.data_ptr()
                d["host_" + name] = host.data_ptr()
        return d

    def resident_rows(self) -> int:
        return int((self.slot2row >= 0).sum())

    def flush(self) -> None:
        """Write every resident row (+ state) back to the host arrays (synchronous)."""
        slots = torch.nonzero(self.slot2row >= 0).flatten()
        if slots.numel() == 0:
            return
        rows = self.slot2row[slots].cpu()
        self.w.index_copy_(0, rows, self.cache_w.index_select(0, slots).cpu())
        for cache, host in ((self.cache_row, self.h_row), (self.cache_m, self.h_m), (self.cache_v, self.h_v)):
            if cache is not None:
                host.index_copy_(0, rows, cache.index_select(0, slots).cpu())


class HostTier:
    """Placement driver for the host-tier shards one rank owns (every rank launches it: barrier)."""

    def __init__(self, coll, *, seed: int = 0, flag_slot: int = 0, flags=None):
        self.coll = coll
        self.shards = [HostShard(coll, i, seed) for i, s in enumerate(coll.shards) if s.slot_map_off >= 0]
        dev = coll.device
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)
        self.flags, self.flag_slot = flags, flag_slot
        self._params = None

    def _build(self) -> dict:
        c = self.coll
        d = {"tables": [hs.params() for hs in self.shards], "world": c.world, "rank": c.rank, "Bl": c.B,
             "peer_offsets": c._peer["offsets"].data_ptr(), "peer_values": c._peer["values"].data_ptr(),
             "step_ptr": self.step_dev.data_ptr(), "block_counter": self.counters.data_ptr(),
             "block_counter2": self.counters.data_ptr() + 4, "status": c.status.ptr, "timeout_ns": c.timeout_ns,
             "grid": c.grid}
        if c.world > 1:
            d.update(flags_local=self.flags.local_ptr, peer_flags=self.flags.peer_ptrs.data_ptr(),
                     flag_in=self.flags.slots(self.flag_slot), epoch_ctr=self.flags.epoch_ptr(self.flag_slot))
            d["block_counter"] = self.flags.block_counter_ptr(self.flag_slot)
        return d

    def prepare(self) -> None:
        """Make every row of the batch in the exchange buffers resident (launches on the current stream)."""
        if self._params is None:
            self._params = self._build()
        native().increment_counter(self.step_dev.data_ptr())
        native().tier_prepare(self._params)

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

    def stats(self) -> dict:
        return {"resident_rows": sum(hs.resident_rows() for hs in self.shards),
                "cache_rows": sum(hs.C for hs in self.shards), "host_bytes": self.host_bytes()}


__all__ = ["HostShard", "HostTier"]
