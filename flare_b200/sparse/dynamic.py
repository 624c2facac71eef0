"""Dynamic (hash-keyed) embedding tables: insert on first sight, CLOCK eviction.

A table spec with ``dynamic=True`` takes any non-negative int32 key; its
``num_embeddings`` rows are HBM slots and a device open-addressing hash map
(``hash_buckets``, a power of two >= 2x the slots) maps keys to slots.
``DynamicTables.prepare`` (called by the collection at the start of every
forward, on every rank) runs the insert / fill / remap kernels
(``csrc/dynamic_emb.cu``): new keys get a slot (evicting the least recently
used one when full) and a row initialised uniform(-init_scale, init_scale)
from a hash of (seed, key, column); the fused forward then reads the slots
from the remap buffers.  ``maintain()`` (host, outside CUDA graphs) rebuilds
the hash map when evictions have left too many tombstones.

This is the reference store's ``lookup_or_insert`` behaviour
(src/flare/runtime/fluxway/workers/dynamic_embedding.py:134-260); the
reference scores rows by frequency (LFU), eviction here is least-recently-used.
"""
from __future__ import annotations

import numpy as np
import torch

from .._native import native

INT_MIN = -(1 << 31)
MASK64 = (1 << 64) - 1


def uniform_init_reference(seed: int, key: int, col: int) -> float:
    """Host restatement of the device init hash (SplitMix64 finaliser) -> uniform [0, 1)."""
    z = (seed + 0x9E3779B97F4A7C15 * ((key & 0xFFFFFFFF) * 4096 + col + 1)) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    z ^= z >> 31
    return float(np.float32((z >> 40) * (1.0 / 16777216.0)))


class DynamicShard:
    def __init__(self, coll, i: int, seed: int):
        s = coll.shards[i]
        self.coll, self.i, self.shard = coll, i, s
        self.C = s.storage_rows
        H = s.spec.hash_buckets or 1 << max(1, (4 * self.C - 1).bit_length())
        if H & (H - 1) or H < 2 * self.C:
            raise ValueError("hash_buckets must be a power of two >= 2 x capacity")
        self.H = H
        dev = coll.device
        self.seed = (seed * 1_000_003 + s.table * 7919) & 0x7FFFFFFF
        self.keys = torch.full((H,), -1, dtype=torch.int32, device=dev)
        self.slot_of = torch.full((H,), -1, dtype=torch.int32, device=dev)
        self.bucket_of = torch.full((self.C,), -1, dtype=torch.int32, device=dev)
        self.stamp = torch.full((self.C,), INT_MIN, dtype=torch.int32, device=dev)
        self.hand = torch.zeros(1, dtype=torch.int32, device=dev)
        self.new_cap = coll.world * coll.stage_cap
        self.new_buckets = torch.empty(self.new_cap, dtype=torch.int32, device=dev)
        self.num_new = torch.zeros(1, dtype=torch.int32, device=dev)
        self.num_tomb = torch.zeros(1, dtype=torch.int32, device=dev)
        self.f = coll.shard_fields(i)

    def params(self) -> dict:
        f = self.f
        d = {"feature": self.coll.features.index(self.shard.spec.feature_name), "ncols": self.shard.ncols,
             "col_begin": self.shard.col_begin, "C": self.C, "H": self.H,
             "init_scale": float(self.shard.spec.init_scale), "seed": self.seed, "keys": self.keys.data_ptr(),
             "slot_of": self.slot_of.data_ptr(), "bucket_of": self.bucket_of.data_ptr(),
             "stamp": self.stamp.data_ptr(), "hand": self.hand.data_ptr(), "weights": f["weight"].data_ptr(),
             "new_buckets": self.new_buckets.data_ptr(), "num_new": self.num_new.data_ptr(),
             "new_cap": self.new_cap, "num_tomb": self.num_tomb.data_ptr()}
        for name, key in (("state_row", "state_row"), ("state_m", "state_m"), ("state_v", "state_v"),
                          ("score", "score")):
            if key in f:
                d[name] = f[key].data_ptr()
        return d

    def live(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(keys, slots) of every resident key."""
        b = self.bucket_of
        ok = b >= 0
        slots = torch.nonzero(ok).flatten().to(torch.int32)
        return self.keys[b[ok].long()], slots

    def rebuild(self) -> None:
        keys, slots = self.live()
        keys, slots = keys.contiguous(), slots.contiguous()
        self.keys.fill_(-1)
        self.slot_of.fill_(-1)
        self.bucket_of.fill_(-1)
        native().dyn_rebuild(self.keys.data_ptr(), self.slot_of.data_ptr(), self.bucket_of.data_ptr(), self.H,
                             keys.data_ptr(), slots.data_ptr(), int(keys.numel()))
        self.num_tomb.zero_()


class DynamicTables:
    """Placement driver for the dynamic shards one rank owns (every rank launches it: barrier)."""

    def __init__(self, coll, *, seed: int, flag_slot: int, flags):
        self.coll = coll
        self.shards = [DynamicShard(coll, i, seed) for i, s in enumerate(coll.shards) if s.dynamic]
        dev = coll.device
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)
        self.flags, self.flag_slot = flags, flag_slot
        self._params = None

    def _build(self) -> dict:
        c = self.coll
        d = {"tables": [s.params() for s in self.shards], "world": c.world, "rank": c.rank, "Bl": c.B,
             "peer_offsets": c._peer["offsets"].data_ptr(), "peer_values": c._peer["values"].data_ptr(),
             "peer_remap": c._peer["remap"].data_ptr(), "step_ptr": self.step_dev.data_ptr(),
             "block_counter": self.counters.data_ptr(), "block_counter2": self.counters.data_ptr() + 4,
             "status": c.status.ptr, "timeout_ns": c.timeout_ns, "grid": c.grid}
        if c.world > 1:
            d.update(flags_local=self.flags.local_ptr, peer_flags=self.flags.peer_ptrs.data_ptr(),
                     flag_in=self.flags.slots(self.flag_slot), epoch_ctr=self.flags.epoch_ptr(self.flag_slot),
                     block_counter=self.flags.block_counter_ptr(self.flag_slot))
        return d

    def prepare(self) -> None:
        if self._params is None:
            self._params = self._build()
        native().increment_counter(self.step_dev.data_ptr())
        native().dyn_prepare(self._params)

    def maintain(self, max_tomb_frac: float = 0.25) -> int:
        """Rebuild hash maps whose tombstones exceed ``max_tomb_frac`` of the buckets (host sync)."""
        n = 0
        for s in self.shards:
            if int(s.num_tomb.item()) > max_tomb_frac * s.H:
                s.rebuild()
                n += 1
        return n

    def resident_keys(self) -> int:
        return sum(int((s.bucket_of >= 0).sum()) for s in self.shards)


__all__ = ["DynamicShard", "DynamicTables", "uniform_init_reference"]
