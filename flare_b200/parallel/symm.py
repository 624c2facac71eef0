"""Symmetric device memory across the ranks of one node.

Each rank makes one raw device allocation; CUDA IPC handles are exchanged with
``all_gather_object`` so every rank maps every peer's allocation (NVLink peer
access through NVSwitch).  Buffers are carved out of the allocation with a
deterministic bump allocator, so buffer k sits at the same offset on every
rank and its peer addresses are ``peer_base[s] + offset``.  The fused kernels
read and write peer buffers directly (P2P loads/stores), and signal through a
flag region in the same heap.

No TMA load with cluster multicast ever reads this memory (it can be another
GPU's memory); kernels use plain loads/stores on it.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .._native import native
from .dist import all_gather_object

ALIGN = 256


@dataclass
class SymBuffer:
    """A buffer at the same heap offset on every rank."""

    local: torch.Tensor
    offset: int
    peer_ptrs: list[int]

    def peer_ptr_tensor(self, device) -> torch.Tensor:
        return torch.tensor(self.peer_ptrs, dtype=torch.int64, device=device)


class SymmetricHeap:
    def __init__(self, nbytes: int, *, rank: int = 0, world_size: int = 1, device: torch.device | None = None):
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.rank, self.world_size = rank, world_size
        self.nbytes = int(nbytes)
        C = native()
        self.base = C.dev_malloc(self.nbytes)
        self._opened: list[int] = []
        if world_size > 1:
            handles = all_gather_object((rank, C.ipc_get_handle(self.base)))
            self.peer_base = [0] * world_size
            for r, h in handles:
                if r == rank:
                    self.peer_base[r] = self.base
                else:
                    p = C.ipc_open_handle(h)
                    self._opened.append(p)
                    self.peer_base[r] = p
        else:
            self.peer_base = [self.base]
        self.offset = 0

    def alloc(self, shape, dtype: torch.dtype) -> SymBuffer:
        """Carve a buffer at the same offset on every rank.

        Every rank must call ``alloc`` in the same order; the reserved size is
        the maximum requested over ranks, so per-rank differences in the
        requested size (e.g. capacities derived from local data) can never
        shift later buffers out of alignment across ranks.
        """
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        reserve = nbytes
        if self.world_size > 1:
            sizes = all_gather_object(int(nbytes))
            reserve = max(sizes)
        off = (self.offset + ALIGN - 1) // ALIGN * ALIGN
        if off + reserve > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted: need {off + reserve} of {self.nbytes} bytes")
        self.offset = off + reserve
        t = native().tensor_from_ptr(self.base + off, list(shape), dtype, self.device.index)
        return SymBuffer(t, off, [b + off for b in self.peer_base])

    def close(self) -> None:
        C = native()
        for p in self._opened:
            C.ipc_close_handle(p)
        self._opened.clear()
        if self.base:
            C.dev_free(self.base)
            self.base = 0

    def __del__(self):  # pragma: no cover - best effort at interpreter exit
        try:
            if getattr(self, "base", 0):
                self.close()
        except Exception:
            pass


class FlagRegion:
    """Barrier flag slots in symmetric memory plus local epoch/counter words.

    ``slots(k)`` returns the uint32 offset of slot-array k (``world_size``
    entries each, peer s writes entry s).  Epoch counters and block counters
    are per barrier user and live in ordinary device memory.
    """

    def __init__(self, heap: SymmetricHeap, num_arrays: int):
        self.heap = heap
        self.world_size = heap.world_size
        self.buf = heap.alloc((num_arrays * heap.world_size,), torch.int32)
        self.buf.local.zero_()
        self.peer_ptrs = torch.tensor(self.buf.peer_ptrs, dtype=torch.int64, device=heap.device)
        self.counters = torch.zeros(2 * num_arrays, dtype=torch.int32, device=heap.device)

    def slots(self, k: int) -> int:
        return k * self.world_size

    @property
    def local_ptr(self) -> int:
        return self.buf.local.data_ptr()

    def epoch_ptr(self, k: int) -> int:
        return self.counters.data_ptr() + 8 * k

    def block_counter_ptr(self, k: int) -> int:
        return self.counters.data_ptr() + 8 * k + 4


__all__ = ["FlagRegion", "SymBuffer", "SymmetricHeap"]
