"""Sharded embedding-bag collection over the GPUs' HBM with fused all-to-alls.

This is the B200 replacement of the reference's sparse-embedding role
(DynamicSparseEmbeddingSPMD, src/flare/runtime/fluxway/workers/
dynamic_embedding.py:134-716) together with the compute-side pooled gather /
scatter (recipes/recsys/ranking/workers/train_worker.py:271-553).  Instead of
routing ids and values between Ray roles, every rank owns the shards given by
the sharding plan and one launch per direction does the exchange in-kernel:

* ``forward()``: every owner reads the ids of each rank's local batch straight
  from that rank's input buffer (NVLink P2P), gathers and pools its HBM rows
  in fp32 and writes the pooled rows straight into the requesting rank's
  pooled-output buffer.
* ``backward()``: every owner pulls the pooled gradients of its columns from
  each rank, deduplicates ids, reduces per row in fp32 and applies the
  row-wise optimizer in place (the gradient never materialises as a dense
  table gradient).

Input layout (per rank, "keyed jagged"): ``offsets`` int32 ``[F*B+1]`` and
``values`` int32 ids, feature-major: the ids of feature f for sample b are
``values[offsets[f*B+b]:offsets[f*B+b+1]]``.  Ids index rows of the table
directly (static vocabulary); negative ids are padding and are skipped.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from .._native import PEER_TIMEOUT_NS, DeviceStatus, dtype_code, native
from ..ops.dense import init_uniform_
from ..parallel.symm import FlagRegion, SymmetricHeap
from .config import SparseOptimizerConfig, SparseTableSpec
from .planner import ShardingPlan, plan_sharding
from .precision import TORCH_DTYPES

# ShardDesc layout shared with embedding.cuh (80 bytes)
_SHARD_DTYPE = np.dtype([
    ("feature", "<i4"), ("col_begin", "<i4"), ("ncols", "<i4"), ("out_col", "<i4"),
    ("rows", "<i8"), ("weight_off", "<i8"), ("row_base", "<i8"),
    ("pooling", "<i4"), ("flags", "<i4"), ("id_rows", "<i8"), ("slot_map_off", "<i8"),
    ("rw_n", "<i4"), ("rw_idx", "<i4"), ("part_col", "<i4"), ("pad", "<i4"),
])
assert _SHARD_DTYPE.itemsize == 80
# RwTable (embedding.cuh): out_col, part_col, ncols, rw_n
_RW_DTYPE = np.dtype([("out_col", "<i4"), ("part_col", "<i4"), ("ncols", "<i4"), ("rw_n", "<i4")])

FLAG_FWD_IN, FLAG_FWD_OUT, FLAG_BWD_IN, FLAG_TIER, FLAG_DYN, NUM_FLAG_ARRAYS = 0, 1, 2, 3, 4, 5


def _with_opt(t: SparseTableSpec, opt: SparseOptimizerConfig) -> SparseTableSpec:
    from dataclasses import replace

    return replace(t, optimizer=opt)


@dataclass
class LocalShard:
    table: int
    spec: SparseTableSpec
    col_begin: int
    ncols: int
    out_col: int
    weight_off: int
    row_base: int
    storage_rows: int = 0      # rows held in HBM (= num_embeddings, or the cache slots of a host-tier table)
    slot_map_off: int = -1     # offset of the row -> slot map of a host-tier table, -1 if resident
    dynamic: bool = False      # hash-keyed table: ids reach the kernels as slots through the remap buffers
    row_index: int = 0         # row-wise piece: holds table rows i with i % row_shards == row_index
    row_shards: int = 1
    part_col: int = -1         # row-wise piece: column of its fp32 partial sums in the partial rows

    @property
    def row_slice(self) -> slice:
        """Rows of the whole table this shard holds, in local order."""
        return slice(self.row_index, None, self.row_shards)


class ShardedEmbeddingBagCollection:
    def __init__(
        self,
        tables: list[SparseTableSpec],
        batch_size: int,
        *,
        max_bag_size: int,
        rank: int = 0,
        world_size: int = 1,
        device: torch.device | None = None,
        heap: SymmetricHeap | None = None,
        plan: ShardingPlan | None = None,
        optimizer: SparseOptimizerConfig | None = None,
        seed: int = 0,
        out_dtype: torch.dtype = torch.bfloat16,
        grad_dtype: torch.dtype = torch.bfloat16,
        light_max: int = 16,
        values_capacity: int | None = None,
        timeout_ns: int = PEER_TIMEOUT_NS,
        init: bool = True,
        deterministic: bool | None = None,
        pipelined: bool = False,
        validate_inputs: bool | None = None,
        accumulation_steps: int = 1,
        pipeline_depth: int = 1,
    ):
        if not tables:
            raise ValueError("at least one table is required")
        self.tables = list(tables)
        self.features = [t.feature_name for t in tables]
        if len(set(self.features)) != len(self.features):
            raise ValueError("every table must read a distinct feature")
        vdt = {t.value_dtype for t in tables}
        if len(vdt) != 1:
            raise ValueError("all tables of one collection share a value dtype")
        self.value_dtype = TORCH_DTYPES[vdt.pop()]
        self.optimizer = optimizer or tables[0].optimizer
        self.B = int(batch_size)
        self.F = len(tables)
        self.rank, self.world = rank, world_size
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        if plan is None:
            tabs = [t if t.optimizer == self.optimizer else _with_opt(t, self.optimizer) for t in self.tables]
            plan = plan_sharding(tabs, world_size)
        self.plan = plan
        self.total_dim = self.plan.total_dim
        self.max_bag = int(max_bag_size)
        self.light_max = int(light_max)
        self.timeout_ns = int(timeout_ns)
        self.out_dtype, self.grad_dtype = out_dtype, grad_dtype
        self.step = 0
        dev = self.device
        # pipelined sparse policy: the backward of step t-d runs after the forward of step t, so the
        # buffers a forward fills for its backward (staged ids / bags / lengths, pooled gradients) rotate
        # over d + 1 slots and every call names its staging slot
        self.pipelined = bool(pipelined)
        if int(pipeline_depth) < 1:
            raise ValueError("pipeline_depth must be >= 1")
        # debug mode (FLARE_VALIDATE_INPUTS=1): every batch's offsets and ids are checked before the copy
        self.validate_inputs = (os.environ.get("FLARE_VALIDATE_INPUTS", "0") == "1" if validate_inputs is None
                                else bool(validate_inputs))
        self.nbuf = int(pipeline_depth) + 1 if self.pipelined else 1
        self._slot = 0
        if self.pipelined and any(t.dynamic or t.cache_rows is not None for t in self.tables):
            raise ValueError("the pipelined sparse policy needs resident static tables: the next forward's "
                             "placement (host tier, dynamic insert) could move a row the pending update writes")
        # gradient-accumulation window: every training forward appends its staging to the window's, and
        # one backward per window reduces all micro-steps' gradients per row in fp32 and applies the
        # optimizer once with the sum scaled by 1 / micro-steps (lookups inside a window see the weights
        # of the window's start)
        self.accum = int(accumulation_steps)
        if self.accum < 1:
            raise ValueError("accumulation_steps must be >= 1")
        if self.accum > 1 and (self.pipelined or any(t.dynamic or t.cache_rows is not None for t in self.tables)):
            raise ValueError("accumulation windows need resident static tables and the synchronous policy: a "
                             "placement inside the window could move a row that an earlier micro-step staged")
        self.micro_filled = 0   # micro-steps staged in the open window
        self._micro = 0         # micro-step of the last training forward

        # ---- row-wise tables: fp32 partial-sum columns (every requester adds the pieces' partials) ----
        self.rw_part_col: dict[int, int] = {}
        pc = 0
        for ti, t in enumerate(self.tables):
            if self.plan.row_shards(ti) > 1:
                if t.dynamic or t.cache_rows is not None:
                    raise ValueError(f"table {t.name}: row-wise pieces are for resident static tables")
                self.rw_part_col[ti] = pc
                pc += t.embedding_dim
        self.part_total = pc
        self.rw_slots = max([self.plan.row_shards(ti) for ti in self.rw_part_col], default=0)

        # ---- local shards ----
        self.shards: list[LocalShard] = []
        woff = 0
        rbase = 0
        smoff = 0
        for p in self.plan.for_rank(rank):
            spec = self.tables[p.table]
            cached = spec.cache_rows is not None
            srows = int(spec.cache_rows) if cached else p.num_rows(spec.num_embeddings)
            part_col = self.rw_part_col[p.table] + p.col_begin if p.row_shards > 1 else -1
            self.shards.append(LocalShard(p.table, spec, p.col_begin, p.ncols, self.plan.out_cols[p.table] + p.col_begin,
                                          woff, rbase, srows, smoff if cached else -1, bool(spec.dynamic),
                                          p.row_index, p.row_shards, part_col))
            woff += srows * p.ncols
            rbase += srows
            if cached:
                smoff += spec.num_embeddings
        self.num_local_elems, self.num_local_rows = woff, rbase
        for p in self.plan.placements:
            t = self.tables[p.table]
            if t.dynamic and p.ncols != t.embedding_dim:
                raise ValueError(f"dynamic table {t.name} cannot be split by columns (one hash map per table)")
        # host-tier tables reach their HBM cache slots through a device row -> slot map (-1 = not resident)
        self.slot_map = torch.full((max(smoff, 1),), -1, dtype=torch.int32, device=self.device) if smoff else None
        self.ncols_max = max([s.ncols for s in self.shards], default=4)
        self.vec = 2 if self.ncols_max > 128 else 1
        gsize = torch.empty(0, dtype=grad_dtype).element_size()
        for s in self.shards:
            if (s.ncols * gsize) % 16:
                raise ValueError(f"shard width {s.ncols}: pooled-gradient rows must be a multiple of 16 bytes")
            g = s.ncols // (4 * self.vec)
            if g < 1 or g > 32 or (g & (g - 1)):
                raise ValueError(f"shard width {s.ncols} unsupported with vec={self.vec}")

        # TMA bulk-gather forward (opt-in, FLARE_EMB_BULK=1): every owned row 16-byte aligned, <= 1 KB.
        # It measured 2x slower than the register-gather forward on the DLRM benchmark (one warp's
        # job chain of id load -> copy issue -> consume is latency bound with 8 warps per SM).
        esize = torch.empty(0, dtype=self.value_dtype).element_size()
        rbytes = [s.ncols * esize for s in self.shards]
        self.bulk = (os.environ.get("FLARE_EMB_BULK", "0") == "1" and
                     all(rb % 16 == 0 and rb <= 1024 and (s.weight_off * esize) % 16 == 0
                         for s, rb in zip(self.shards, rbytes)))
        self.bulk_vec = 2 if max(rbytes, default=16) > 512 else 1

        desc = np.zeros(max(len(self.shards), 1), dtype=_SHARD_DTYPE)
        for i, s in enumerate(self.shards):
            desc[i] = (self.features.index(s.spec.feature_name), s.col_begin, s.ncols, s.out_col,
                       s.storage_rows, s.weight_off, s.row_base, 1 if s.spec.pooling == "mean" else 0,
                       1 if s.dynamic else 0, s.spec.num_embeddings, s.slot_map_off, s.row_shards, s.row_index,
                       s.part_col, 0)
        self.shard_desc = torch.from_numpy(desc.view(np.uint8).copy()).to(dev)
        rw = np.zeros(max(len(self.rw_part_col), 1), dtype=_RW_DTYPE)
        for k, (ti, pcol) in enumerate(sorted(self.rw_part_col.items())):
            rw[k] = (self.plan.out_cols[ti], pcol, self.tables[ti].embedding_dim, self.plan.row_shards(ti))
        self.rw_desc = torch.from_numpy(rw.view(np.uint8).copy()).to(dev)

        # ---- parameters and optimizer state (local HBM) ----
        self.weights = torch.empty(max(woff, 4), dtype=self.value_dtype, device=dev)
        if init:
            for s in self.shards:
                n = s.storage_rows * s.ncols
                view = self.weights[s.weight_off:s.weight_off + n]
                stream_seed = (seed * 1_000_003 + s.table * 7919) & 0x7FFFFFFF
                init_uniform_(view, -s.spec.init_scale, s.spec.init_scale, stream_seed, ncols=s.ncols,
                              dim=s.spec.embedding_dim, col_begin=s.col_begin, row_stride=s.row_shards,
                              row_first=s.row_index)
        opt = self.optimizer
        z32 = lambda n: torch.zeros(max(n, 4), dtype=torch.float32, device=dev)  # noqa: E731
        self.state_row = z32(rbase) if opt.needs_row_state else None
        self.state_m = z32(woff) if opt.needs_m else None
        self.state_v = z32(woff) if opt.needs_v else None
        self.score = z32(rbase) if opt.needs_score else None
        self.lut = (torch.tensor(opt.custom_lut, dtype=torch.float32, device=dev)
                    if opt.dynamic_lr_policy == "custom_lut" else None)

        # rows updated since the last checkpoint (incremental sparse saves): one bit per local row
        self.dirty_bits = torch.zeros(max((rbase + 31) // 32, 1), dtype=torch.int32, device=dev)

        # ---- staging ----
        ns = max(len(self.shards), 1)
        self.stage_cap = self.B * self.max_bag
        nslot = ns * world_size
        self._stages = [dict(ids=torch.empty(nslot * self.stage_cap, dtype=torch.int32, device=dev),
                             bag=torch.empty(nslot * self.stage_cap, dtype=torch.int32, device=dev),
                             count=torch.zeros(nslot, dtype=torch.int32, device=dev),
                             len=torch.zeros(nslot * self.B, dtype=torch.int32, device=dev))
                        for _ in range(self.nbuf)]
        st0 = self._stages[0]
        self.stage_ids, self.stage_bag, self.stage_count, self.stage_len = st0["ids"], st0["bag"], st0["count"], st0["len"]
        # multi-GPU: local copies of every (shard, source) offset run (ids go to stage_ids) fetched in bulk
        # before the forward (FLARE_EMB_FETCH=0 reads them from the peers inside the forward instead)
        self.fetch = world_size > 1 and os.environ.get("FLARE_EMB_FETCH", "1") != "0"
        self.fetch_offs = (torch.zeros(nslot * (self.B + 1), dtype=torch.int32, device=dev)
                           if self.fetch else None)
        # the backward's batch: one step, or every micro-step of an accumulation window
        self.Bb = self.B * self.accum
        self.bwd_cap = self.stage_cap * self.accum
        self.nslot = nslot
        self._win = None
        if self.accum > 1:
            i32z = lambda n: torch.zeros(n, dtype=torch.int32, device=dev)  # noqa: E731
            self._win = dict(ids=i32z(nslot * self.bwd_cap), bag=i32z(nslot * self.bwd_cap),
                             prefix=i32z((self.accum + 1) * nslot), len=i32z(nslot * self.Bb))
        self.stage_rank = torch.empty(nslot * self.bwd_cap, dtype=torch.int32, device=dev)
        self.slot_start = torch.zeros(nslot + 1, dtype=torch.int32, device=dev)
        self.grad_stage_ld = self.ncols_max
        self.max_occ = nslot * self.bwd_cap
        self.flags_occ = torch.empty(self.max_occ, dtype=torch.int32, device=dev)
        self.num_unique = torch.zeros(8, dtype=torch.int32, device=dev)
        self.seg_start = torch.empty(self.max_occ + 1, dtype=torch.int32, device=dev)
        self.occ = torch.empty(self.max_occ, dtype=torch.int32, device=dev)
        # deterministic-reduction mode (FLARE_DETERMINISTIC=1): rows add their occurrences in staging
        # order, so repeated runs are bitwise identical (a race detector for the sparse backward)
        if deterministic is None:
            deterministic = os.environ.get("FLARE_DETERMINISTIC", "0") == "1"
        self.deterministic = bool(deterministic)
        # hash-dedup backward (default): the step's touched rows go into an open-addressing table that
        # stays in L2; the sorted per-row path serves the deterministic mode (and FLARE_EMB_LEGACY_BWD=1)
        # (its lanes cover 16 columns: every shard width a multiple of 16)
        self.hash_bwd = (not self.deterministic and os.environ.get("FLARE_EMB_LEGACY_BWD", "0") != "1"
                         and rbase < 2**32 - 1 and all(sh.ncols % 16 == 0 for sh in self.shards))
        i32 = lambda n: torch.empty(max(int(n), 4), dtype=torch.int32, device=dev)  # noqa: E731
        # pooled gradients pulled from every rank (at one GPU the hash path reads them where the dense
        # backward wrote them)
        # (16-byte gradient loads need 8-element-aligned rows for bf16 gradients)
        aligned = grad_dtype == torch.float32 or (self.total_dim % 8 == 0 and all(sh.out_col % 8 == 0
                                                                                 for sh in self.shards))
        self.grad_direct = (self.hash_bwd and world_size == 1 and aligned
                            and os.environ.get("FLARE_EMB_GRAD_STAGE", "0") != "1")
        staged = not self.grad_direct
        self.grad_stage = torch.empty(nslot * self.Bb * self.ncols_max if staged else 8, dtype=grad_dtype, device=dev)
        if self.hash_bwd:
            # touched-row table: a region sized for the step's unique rows (its slots are prefetched into L2
            # and take every key's first probes) and an overflow table with room for every possible key
            hcap = 1 << max(4, (self.max_occ - 1).bit_length())
            self.hash_region_cap = min(hcap, 1 << 22)
            tiles, max_chunks, max_parts, scan_vals = native().emb_hash_sizes(self.max_occ, self.light_max)
            # slot word: key (low 32 bits) = 0xFFFFFFFF and count 0 when empty; every backward leaves it empty
            self.htab = torch.full((self.hash_region_cap + hcap,), 0xFFFFFFFF, dtype=torch.int64, device=dev)
            self.hash = dict(hcap=hcap, hregion=self.hash_region_cap, max_tiles=tiles, max_chunks=max_chunks,
                             max_parts=max_parts, hseg=i32(self.hash_region_cap + hcap),
                             ovf_list=i32(self.max_occ), occ_bag=i32(self.max_occ),
                             lrec=i32(4 * self.max_occ), crec=i32(8 * max_chunks),
                             hpart=torch.empty(max_parts * self.ncols_max, dtype=torch.float32, device=dev),
                             occ_scale=(torch.empty(self.max_occ, dtype=torch.float32, device=dev)
                                        if any(s.spec.pooling == "mean" for s in self.shards) else None),
                             scan_val=torch.zeros(tiles * scan_vals, dtype=torch.int32, device=dev))
        else:
            self.htab, self.hash = None, None
            # per-row dedup scratch (returns to zero after every backward)
            self.row_count = torch.zeros(max(rbase, 4), dtype=torch.int32, device=dev)
            self.row2u = torch.zeros(max(rbase, 4), dtype=torch.int32, device=dev)
            self.pos = i32(self.max_occ + 1)
            self.uniq_row = torch.empty(self.max_occ, dtype=torch.int64, device=dev)
            self.uniq_shard = i32(self.max_occ)
            self.cnt_u = i32(self.max_occ)
            self.first_gidx = i32(self.max_occ)
            self.block_sums = i32(512)
            # rows with more than light_max occurrences take the chunked path
            self.max_heavy = min(self.max_occ // (self.light_max + 1) + 1, 1 << 20)
            self.heavy = i32(self.max_heavy)
            self.heavy_start = i32(self.max_heavy + 1)
            self.hcnt = i32(self.max_heavy)
            # one fp32 partial row per (heavy row, 256-occurrence chunk) segment
            self.heavy_acc = torch.zeros((self.max_heavy + self.max_occ // 256 + 2) * 128 * self.vec,
                                         dtype=torch.float32, device=dev)
        self.det = None
        if self.deterministic:
            nbytes = int(native().emb_det_temp_bytes(self.max_occ))
            self.det = dict(first=torch.full((max(rbase, 4),), 2**31 - 1, dtype=torch.int32, device=dev),
                            keys=torch.empty(2 * self.max_occ, dtype=torch.int32, device=dev),
                            vals=torch.empty(self.max_occ, dtype=torch.int32, device=dev),
                            temp=torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev), bytes=nbytes)

        # ---- exchange buffers (symmetric when distributed) ----
        self.values_capacity = int(values_capacity or self.F * self.B * self.max_bag)
        if heap is None:
            if world_size > 1:
                raise ValueError("a SymmetricHeap is required for world_size > 1")
            heap = SymmetricHeap(self._heap_bytes(), device=dev)
            self._own_heap = heap
        else:
            self._own_heap = None
        self.heap = heap
        self.in_offsets = heap.alloc((self.F * self.B + 1,), torch.int32)
        self.in_values = heap.alloc((self.values_capacity,), torch.int32)
        self.pooled = heap.alloc((self.B, self.total_dim), out_dtype)
        self.grad_ins = [heap.alloc((self.Bb, self.total_dim), grad_dtype) for _ in range(self.nbuf)]
        self.grad_in = self.grad_ins[0]
        self.flags = FlagRegion(heap, NUM_FLAG_ARRAYS)
        any_dynamic = any(t.dynamic for t in self.tables)
        # dynamic tables: owners write each occurrence's slot into the requester's remap buffer
        self.remap = heap.alloc((self.values_capacity,), torch.int32) if any_dynamic else None
        # row-wise tables: owners write fp32 partial pooled rows [residue][sample][part col] into the requester
        self.partials = (heap.alloc((self.rw_slots, self.B, self.part_total), torch.float32)
                         if self.rw_part_col else None)
        self._peer = {
            "offsets": self.in_offsets.peer_ptr_tensor(dev),
            "values": self.in_values.peer_ptr_tensor(dev),
            "out": self.pooled.peer_ptr_tensor(dev),
        }
        self._peer_grad = [g.peer_ptr_tensor(dev) for g in self.grad_ins]
        if self.remap is not None:
            self._peer["remap"] = self.remap.peer_ptr_tensor(dev)
        if self.partials is not None:
            self._peer["part"] = self.partials.peer_ptr_tensor(dev)
        self.status = DeviceStatus(dev)
        self.grid = native().device_sm_count() * 8
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=dev)  # device-resident optimizer step
        # host-DRAM tier: placement kernels run before every forward (on every rank when any table is
        # host-tier, because the placement kernel's barrier spans all ranks)
        self.host_tier = None
        if any(t.cache_rows is not None for t in self.tables):
            from .host_tier import HostTier

            self.host_tier = HostTier(self, seed=seed, flag_slot=FLAG_TIER, flags=self.flags)
        self.dynamic = None
        if any_dynamic:
            from .dynamic import DynamicTables

            self.dynamic = DynamicTables(self, seed=seed, flag_slot=FLAG_DYN, flags=self.flags)

    @staticmethod
    def exchange_bytes(tables: list[SparseTableSpec], batch_size: int, max_bag_size: int,
                       values_capacity: int | None = None, plan: ShardingPlan | None = None,
                       pipelined: bool = False, accumulation_steps: int = 1, pipeline_depth: int = 1) -> int:
        """Symmetric memory of the exchange buffers (ids, pooled rows, pooled grads, row-wise partials)."""
        F, B = len(tables), int(batch_size)
        cap = values_capacity or F * B * max_bag_size
        dim = sum(t.embedding_dim for t in tables)
        shards = [plan.row_shards(i) if plan is not None else t.shards for i, t in enumerate(tables)]
        rw = [i for i, r in enumerate(shards) if r > 1]
        part = 4 * max([shards[i] for i in rw], default=0) * B * sum(tables[i].embedding_dim for i in rw)
        remap = 4 * cap if any(t.dynamic for t in tables) else 0
        grads = (int(pipeline_depth) + 1 if pipelined else 1) * max(1, int(accumulation_steps))
        return 4 * (F * B + 1) + 4 * cap + remap + (1 + grads) * 4 * B * dim + part + NUM_FLAG_ARRAYS * 64 + 4096

    def _heap_bytes(self) -> int:
        b = (self.F * self.B + 1) * 4 + 2 * self.F * self.B * self.max_bag * 4
        b += (self.B + self.nbuf * self.Bb) * self.total_dim * 4 + NUM_FLAG_ARRAYS * 64 + 8 * 256
        b += self.rw_slots * self.B * self.part_total * 4 + 256
        return b + (1 << 20)

    # ------------------------------------------------------------------ API
    @property
    def pooled_output(self) -> torch.Tensor:
        """[B, total_dim] pooled embeddings of this rank's local batch (bf16)."""
        return self.pooled.local

    @property
    def grad_input(self) -> torch.Tensor:
        """[B, total_dim] buffer the dense backward writes the pooled gradients into (slot / micro-step of the
        last training forward)."""
        g = self.grad_ins[self._slot].local
        return g if self.accum == 1 else g[self._micro * self.B:(self._micro + 1) * self.B]

    def _slot_of(self, slot: int | None) -> int:
        s = self._slot if slot is None else int(slot)
        if not 0 <= s < self.nbuf:
            raise ValueError(f"staging slot {s} out of range (the collection has {self.nbuf})")
        return s

    def set_input(self, offsets: torch.Tensor, values: torch.Tensor, non_blocking: bool = True) -> None:
        """Copy this rank's keyed-jagged batch into the exchange buffers."""
        if offsets.numel() != self.F * self.B + 1:
            raise ValueError(f"offsets must have F*B+1 = {self.F * self.B + 1} entries")
        n = values.numel()
        if n > self.values_capacity:
            raise ValueError(f"{n} ids exceed the values capacity {self.values_capacity}")
        if self.validate_inputs:
            validate_keyed_jagged(offsets, values, self.tables, self.B, self.max_bag)
        self.in_offsets.local.copy_(offsets, non_blocking=non_blocking)
        self.in_values.local[:n].copy_(values, non_blocking=non_blocking)

    def forward(self, training: bool = True, slot: int | None = None) -> torch.Tensor:
        """Pooled embeddings of this rank's batch; ``training`` also stages the backward (into ``slot``)."""
        sl = self._slot_of(slot)
        if training:
            self._slot = sl
        st = self._stages[sl]
        d = dict(
            shards=self.shard_desc.data_ptr(), num_shards=len(self.shards), world=self.world, rank=self.rank,
            Bl=self.B, F=self.F, peer_offsets=self._peer["offsets"].data_ptr(),
            peer_values=self._peer["values"].data_ptr(), peer_out=self._peer["out"].data_ptr(),
            out_stride=self.total_dim, weights=self.weights.data_ptr(), w_dtype=dtype_code(self.value_dtype),
            out_dtype=dtype_code(self.out_dtype), vec=self.bulk_vec if self.bulk else self._fwd_vec(),
            bulk=1 if self.bulk else 0, stage_ids=st["ids"].data_ptr(),
            slot_map=self.slot_map.data_ptr() if self.slot_map is not None else 0,
            stage_bag=st["bag"].data_ptr(), stage_count=st["count"].data_ptr(),
            stage_len=st["len"].data_ptr(), stage_cap=self.stage_cap,
            flags_local=self.flags.local_ptr, peer_flags=self.flags.peer_ptrs.data_ptr(),
            flag_in=self.flags.slots(FLAG_FWD_IN), flag_out=self.flags.slots(FLAG_FWD_OUT),
            epoch_ctr=self.flags.epoch_ptr(FLAG_FWD_IN), block_counter=self.flags.block_counter_ptr(FLAG_FWD_IN),
            status=self.status.ptr, timeout_ns=self.timeout_ns, grid=self.grid,
            fwd_minb=int(os.environ.get("FLARE_EMB_FWD_MINB", "4")),
        )
        if self.host_tier is not None:
            self.host_tier.prepare()
        if self.dynamic is not None:
            self.dynamic.prepare()
            d["peer_remap"] = self._peer["remap"].data_ptr()
        if self.fetch and not self.bulk and training:
            d["fetch_offs"] = self.fetch_offs.data_ptr()
        if self.partials is not None:
            d.update(peer_part=self._peer["part"].data_ptr(), part_stride=self.part_total,
                     rw_tables=self.rw_desc.data_ptr(), num_rw=len(self.rw_part_col))
        native().emb_forward(d)
        if training and self.accum > 1:
            k = self.micro_filled
            if k >= self.accum:
                raise RuntimeError(f"the accumulation window holds {self.accum} micro-steps: run backward() first")
            w = self._win
            native().emb_window_append(dict(
                ids=st["ids"].data_ptr(), bag=st["bag"].data_ptr(), count=st["count"].data_ptr(),
                len=st["len"].data_ptr(), wids=w["ids"].data_ptr(), wbag=w["bag"].data_ptr(),
                wprefix=w["prefix"].data_ptr(), wlen=w["len"].data_ptr(), nslot=self.nslot, Bl=self.B,
                micro=k, micro_steps=self.accum, stage_cap=self.stage_cap))
            self._micro, self.micro_filled = k, k + 1
        return self.pooled.local

    def _fwd_vec(self) -> int:
        """float4 vectors per lane in the forward: 2 (8 columns per lane), so a 128-column shard runs two
        bags per warp and each warp keeps two bags' id -> row chains in flight (1.7 % faster per DLRM step
        than one bag per warp); FLARE_EMB_FWD_VEC=1 for one bag per warp up to 128 columns."""
        v = int(os.environ.get("FLARE_EMB_FWD_VEC", "2"))
        if v == 2 and all(sh.ncols % 8 == 0 and (sh.ncols // 8) & (sh.ncols // 8 - 1) == 0 for sh in self.shards):
            return 2
        return self.vec

    def backward(self, step: int | None = None, slot: int | None = None) -> None:
        """Consume the pooled gradients of staging ``slot`` (default: the last forward's) and update the owned shards.

        The optimizer step used for bias corrections is the device counter,
        advanced by one per call (``step`` sets it explicitly first).  With an
        accumulation window the call closes the window: every staged
        micro-step's gradients are summed per row and the optimizer applies
        the sum divided by the number of micro-steps (a shorter tail window
        divides by its own count).
        """
        sl = self._slot_of(slot)
        st = self._stages[sl]
        micro = 1
        if self.accum > 1:
            micro = self.micro_filled
            if micro == 0:
                raise RuntimeError("backward() with no micro-step staged in the accumulation window")
            w = self._win
            st = dict(ids=w["ids"], bag=w["bag"], len=w["len"],
                      count=w["prefix"][micro * self.nslot:(micro + 1) * self.nslot])
            self.micro_filled = 0
        if step is not None:
            self.step = int(step) - 1
            self.step_dev.fill_(self.step)
        self.step += 1
        native().increment_counter(self.step_dev.data_ptr())
        op = self.optimizer.kernel_params(self.step)
        op.update(
            grad_scale=1.0 / micro,
            step_ptr=self.step_dev.data_ptr(),
            state_row=self.state_row.data_ptr() if self.state_row is not None else 0,
            state_m=self.state_m.data_ptr() if self.state_m is not None else 0,
            state_v=self.state_v.data_ptr() if self.state_v is not None else 0,
            score=self.score.data_ptr() if self.score is not None else 0,
            lut=self.lut.data_ptr() if self.lut is not None else 0,
            lut_len=self.lut.numel() if self.lut is not None else 0,
        )
        d = dict(
            shards=self.shard_desc.data_ptr(), num_shards=len(self.shards), world=self.world, rank=self.rank,
            Bl=self.Bb, peer_grad=self._peer_grad[sl].data_ptr(), out_stride=self.total_dim,
            grad_dtype=dtype_code(self.grad_dtype), grad_stage=self.grad_stage.data_ptr(),
            grad_stage_ld=self.grad_stage_ld, stage_ids=st["ids"].data_ptr(),
            stage_bag=st["bag"].data_ptr(), stage_rank=self.stage_rank.data_ptr(),
            slot_start=self.slot_start.data_ptr(),
            stage_count=st["count"].data_ptr(), stage_len=st["len"].data_ptr(),
            stage_cap=self.bwd_cap, weights=self.weights.data_ptr(), w_dtype=dtype_code(self.value_dtype),
            flags=self.flags_occ.data_ptr(), num_unique=self.num_unique.data_ptr(),
            seg_start=self.seg_start.data_ptr(), occ=self.occ.data_ptr(),
            light_max=self.light_max, max_occ=self.max_occ, opt=op, dirty=self.dirty_bits.data_ptr(),
            flags_local=self.flags.local_ptr, peer_flags=self.flags.peer_ptrs.data_ptr(),
            flag_in=self.flags.slots(FLAG_BWD_IN), epoch_ctr=self.flags.epoch_ptr(FLAG_BWD_IN),
            block_counter=self.flags.block_counter_ptr(FLAG_BWD_IN), status=self.status.ptr,
            timeout_ns=self.timeout_ns, ncols_max=self.ncols_max, grid=self.grid,
        )
        if self.hash is not None:
            h = self.hash
            self._tune_hash_region()
            d.update(hash_mode=1, grad_direct=int(self.grad_direct), htab=self.htab.data_ptr(), hcap=h["hcap"],
                     hregion=h["hregion"], hprefetch=0 if os.environ.get("FLARE_EMB_HASH_PREFETCH") == "0" else 1,
                     light_prefetch=1 if os.environ.get("FLARE_EMB_LIGHT_PREFETCH") == "1" else 0,
                     chunk_variant=int(os.environ.get("FLARE_EMB_CHUNK_VARIANT", "1")),
                     occ_h=self.flags_occ.data_ptr(),
                     occ_rank=self.stage_rank.data_ptr(), max_tiles=h["max_tiles"], max_chunks=h["max_chunks"],
                     max_parts=h["max_parts"],
                     occ_scale=h["occ_scale"].data_ptr() if h["occ_scale"] is not None else 0,
                     **{k: h[k].data_ptr() for k in ("hseg", "ovf_list", "occ_bag", "lrec", "crec", "hpart",
                                                     "scan_val")})
        else:
            d.update(row_count=self.row_count.data_ptr(), row2u=self.row2u.data_ptr(), pos=self.pos.data_ptr(),
                     uniq_row=self.uniq_row.data_ptr(), uniq_shard=self.uniq_shard.data_ptr(),
                     cnt_u=self.cnt_u.data_ptr(), first_gidx=self.first_gidx.data_ptr(),
                     block_sums=self.block_sums.data_ptr(), heavy=self.heavy.data_ptr(),
                     heavy_start=self.heavy_start.data_ptr(), hcnt=self.hcnt.data_ptr(),
                     heavy_acc=self.heavy_acc.data_ptr(), max_heavy=self.max_heavy)
        if self.det is not None:
            d.update(deterministic=1, det_first=self.det["first"].data_ptr(), det_keys=self.det["keys"].data_ptr(),
                     det_vals=self.det["vals"].data_ptr(),
                     det_temp=self.det["temp"].data_ptr(), det_temp_bytes=self.det["bytes"])
        native().emb_backward(d)

    def _tune_hash_region(self) -> None:
        """Size the L2 region of the touched-row table from the first backward's unique-row count.

        The first backward runs with the largest region; the next call made outside stream capture
        reads its count (one device sync, during warm-up) and keeps the region at 1.6x that count,
        rounded up to a power of two, for every later step, so a CUDA graph captured after the
        warm-up steps records the tuned region.  Keys beyond the region's probes go to the overflow
        table, so the choice affects speed only."""
        h = self.hash
        if h.get("tuned") or torch.cuda.is_current_stream_capturing():
            return
        if not h.get("ran"):
            h["ran"] = True
            return
        u = int(self.num_unique[0].item())
        if u > 0:
            h["hregion"] = min(self.hash_region_cap, 1 << max(12, int(u * 1.6 - 1).bit_length()))
        h["tuned"] = True

    def dirty_rows(self, row_base: int, rows: int) -> torch.Tensor:
        """Local row indices in [row_base, row_base + rows) updated since the last ``clear_dirty`` (relative
        to ``row_base``, ascending)."""
        if rows <= 0:
            return torch.zeros(0, dtype=torch.int64, device=self.device)
        w0, w1 = row_base // 32, (row_base + rows + 31) // 32
        words = self.dirty_bits[w0:w1].to(torch.int64) & 0xFFFFFFFF
        bits = (words.unsqueeze(1) >> torch.arange(32, device=words.device)) & 1
        flags = bits.reshape(-1)[row_base - 32 * w0:row_base - 32 * w0 + rows]
        return torch.nonzero(flags).flatten()

    @property
    def dirty(self) -> torch.Tensor:
        """Per-row dirty flags (uint8, unpacked from the bitmap)."""
        n = self.num_local_rows
        out = torch.zeros(max(n, 4), dtype=torch.uint8, device=self.device)
        out[self.dirty_rows(0, n)] = 1
        return out

    def clear_dirty(self) -> None:
        self.dirty_bits.zero_()

    def check(self) -> None:
        self.status.check("sharded embedding")

    def last_step_stats(self) -> dict:
        """Unique rows, valid occurrences and heavy rows of the last backward (device sync)."""
        u, t, h = self.num_unique.tolist()[:3]
        return {"unique_rows": u, "occurrences": t, "heavy_rows": h}

    # ------------------------------------------------------------ state I/O
    def shard_view(self, i: int) -> torch.Tensor:
        """HBM rows of shard i (the whole table, or the cache slots of a host-tier table)."""
        s = self.shards[i]
        n = s.storage_rows * s.ncols
        return self.weights[s.weight_off:s.weight_off + n].view(s.storage_rows, s.ncols)

    def row_state_view(self, i: int) -> torch.Tensor | None:
        if self.state_row is None:
            return None
        s = self.shards[i]
        return self.state_row[s.row_base:s.row_base + s.storage_rows]

    def shard_fields(self, i: int) -> dict[str, torch.Tensor]:
        """Device views of shard i: weight [rows, ncols] and optimizer state."""
        s = self.shards[i]
        rows, n = s.storage_rows, s.storage_rows * s.ncols
        out = {"weight": self.shard_view(i)}
        if self.state_row is not None:
            out["state_row"] = self.state_row[s.row_base:s.row_base + rows]
        if self.state_m is not None:
            out["state_m"] = self.state_m[s.weight_off:s.weight_off + n].view(rows, s.ncols)
        if self.state_v is not None:
            out["state_v"] = self.state_v[s.weight_off:s.weight_off + n].view(rows, s.ncols)
        if self.score is not None:
            out["score"] = self.score[s.row_base:s.row_base + rows]
        return out

    def local_state(self) -> dict:
        """Owned shards with optimizer state (host copies), keyed by (table, col_begin, row_index)."""
        out = {}
        for i, s in enumerate(self.shards):
            entry = {"weight": self.shard_view(i).cpu(), "ncols": s.ncols}
            if self.state_row is not None:
                entry["state_row"] = self.row_state_view(i).cpu()
            n = s.storage_rows * s.ncols
            if self.state_m is not None:
                entry["state_m"] = self.state_m[s.weight_off:s.weight_off + n].view(-1, s.ncols).cpu()
            if self.state_v is not None:
                entry["state_v"] = self.state_v[s.weight_off:s.weight_off + n].view(-1, s.ncols).cpu()
            if self.score is not None:
                entry["score"] = self.score[s.row_base:s.row_base + s.storage_rows].cpu()
            out[(s.spec.name, s.col_begin, s.row_index)] = entry
        return out

    def export_pieces(self) -> dict:
        """Host fp32 copies of the owned weights keyed ``(table, col_begin, row_index, row_shards)``."""
        return {(s.table, s.col_begin, s.row_index, s.row_shards): self.shard_view(i).float().cpu()
                for i, s in enumerate(self.shards)}

    @staticmethod
    def assemble_tables(pieces: dict, tables: list[SparseTableSpec]) -> list[torch.Tensor]:
        """Whole tables from the pieces of every rank (``export_pieces`` of each, merged)."""
        out = [torch.zeros(t.num_embeddings, t.embedding_dim) for t in tables]
        for (t, c, r, R), w in pieces.items():
            out[t][r::R, c:c + w.shape[1]] = w
        return out

    def load_local_state(self, state: dict) -> None:
        for i, s in enumerate(self.shards):
            entry = state[(s.spec.name, s.col_begin, s.row_index)]
            self.shard_view(i).copy_(entry["weight"])
            n = s.storage_rows * s.ncols
            if self.state_row is not None and "state_row" in entry:
                self.row_state_view(i).copy_(entry["state_row"])
            if self.state_m is not None and "state_m" in entry:
                self.state_m[s.weight_off:s.weight_off + n].copy_(entry["state_m"].reshape(-1))
            if self.state_v is not None and "state_v" in entry:
                self.state_v[s.weight_off:s.weight_off + n].copy_(entry["state_v"].reshape(-1))
            if self.score is not None and "score" in entry:
                self.score[s.row_base:s.row_base + s.storage_rows].copy_(entry["score"])

    def memory_bytes(self) -> int:
        tensors = [self.weights, self.state_row, self.state_m, self.state_v, self.score, self.stage_ids,
                   self.stage_bag, self.stage_rank, self.grad_stage, self.occ, self.seg_start, self.flags_occ]
        if self.hash is not None:
            tensors += [self.htab] + [v for v in self.hash.values() if isinstance(v, torch.Tensor)]
        else:
            tensors += [self.row_count, self.row2u, self.uniq_row, self.pos, self.cnt_u, self.first_gidx,
                        self.heavy, self.heavy_acc]
        return sum(t.numel() * t.element_size() for t in tensors if t is not None)


def validate_keyed_jagged(offsets: torch.Tensor, values: torch.Tensor, tables: list[SparseTableSpec], batch: int,
                          max_bag: int) -> None:
    """Check a keyed-jagged batch before the kernels see it (debug mode; reads the data on the host).

    ``offsets`` [F*B+1] int32 starts at 0, never decreases and ends at the id count; no bag is longer
    than ``max_bag`` (the staging capacity); every id of table f is in [0, rows_f) (dynamic tables:
    any id >= 0).  Raises ``ValueError`` naming the first offending feature / sample.  The same
    contract as the reference's ragged-input validation before native writes
    (src/flare/data/schema/input.py:90-123)."""
    F = len(tables)
    if offsets.dtype != torch.int32 or values.dtype != torch.int32:
        raise ValueError("offsets and ids must be int32")
    off = offsets.detach().to("cpu", torch.int64)
    if off.numel() != F * batch + 1 or int(off[0]) != 0:
        raise ValueError("offsets must have F*B+1 entries and start at 0")
    lens = off[1:] - off[:-1]
    if bool((lens < 0).any()):
        k = int(torch.nonzero(lens < 0)[0])
        raise ValueError(f"offsets decrease at feature {k // batch}, sample {k % batch}")
    if int(off[-1]) != values.numel():
        raise ValueError(f"offsets end at {int(off[-1])}, but {values.numel()} ids were given")
    if bool((lens > max_bag).any()):
        k = int(torch.nonzero(lens > max_bag)[0])
        raise ValueError(f"feature {k // batch}, sample {k % batch}: bag of {int(lens[k])} ids > max_bag {max_bag}")
    ids = values.detach().to("cpu", torch.int64)
    for f, t in enumerate(tables):
        seg = ids[int(off[f * batch]):int(off[(f + 1) * batch])]
        if seg.numel() == 0:
            continue
        lo, hi = int(seg.min()), int(seg.max())
        if lo < 0 or (not t.dynamic and hi >= t.num_embeddings):
            raise ValueError(f"feature {f} (table {t.name}): ids span [{lo}, {hi}], rows [0, {t.num_embeddings})")


def expected_math_bytes(num_ids: int, dim: int, value_bytes: int = 4) -> float:
    """Bytes a forward gather-pool must read at minimum (for roofline reports)."""
    return float(num_ids) * dim * value_bytes


__all__ = ["LocalShard", "ShardedEmbeddingBagCollection", "expected_math_bytes", "validate_keyed_jagged"]
