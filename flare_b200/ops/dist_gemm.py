"""Fused tensor/FSDP-parallel GEMMs on tcgen05: all-gather -> GEMM, GEMM -> reduce-scatter.

The kernel (``csrc/gemm_dist.cu``) is a persistent, cooperatively launched
tcgen05 GEMM.  Three objects describe what it moves:

* ``ShardedRows`` - a bf16 matrix in symmetric memory whose stored rows are
  split over a group of ranks (member q owns rows ``[q*S, (q+1)*S)``).  Used
  as a GEMM operand it is all-gathered inside the GEMM: copy warps pull the
  peers' row chunks over NVLink into the local buffer while the tensor cores
  work on tiles whose rows are already local.  Activations under
  sequence-parallel tensor parallelism and weights under FSDP both use it.
* ``RowReduceScatter`` - receive buffers and flags for a GEMM whose output
  rows are reduce-scattered over a group: each rank sends bf16 partial tiles
  of the rows a peer owns straight into that peer's memory and sums the
  partials of its own rows in the epilogue.
* ``DistGemmContext`` - the per-process barrier slots, epoch word and status.

``DistGemm`` binds one call site (operands, epilogue, collectives) once; the
call itself is a single kernel launch, so it can be captured in a CUDA graph.

The reference has no tensor parallelism and runs its FSDP (ZeRO-3) gathers as
separate XLA all-gathers (src/flare/jax/training/state/layout.py:176-194).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .._native import DEFAULT_TIMEOUT_NS, PEER_TIMEOUT_NS, DeviceStatus, native

BM, BN = 128, 256
F32, BF16 = 0, 1
PIECE_VECS = 512  # 16-byte vectors (8 KiB) per copy work item of a gathered chunk


def _pieces(chunk_rows: int, cols: int) -> tuple[int, int]:
    """(pieces per chunk, vectors per piece) for a chunk of ``chunk_rows`` rows of ``cols`` bf16."""
    vecs = chunk_rows * (_round_up(cols, 8) // 8)
    per = PIECE_VECS
    while (vecs + per - 1) // per > 4096:
        per *= 2
    return (vecs + per - 1) // per, per


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class DistGemmContext:
    """Barrier slots (symmetric), epoch/counter words and the status word."""

    def __init__(self, heap, *, timeout_ns: int | None = None):
        self.heap = heap
        self.rank, self.world = heap.rank, heap.world_size
        self.device = heap.device
        self.bar = heap.alloc((max(self.world, 1),), torch.int32)
        self.bar.local.zero_()
        self.ctl = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.status = DeviceStatus(self.device)
        self.timeout_ns = int(timeout_ns or (PEER_TIMEOUT_NS if self.world > 1 else DEFAULT_TIMEOUT_NS))

    def fields(self) -> dict:
        return {"world": self.world, "rank": self.rank, "bar_local": self.bar.local.data_ptr(),
                "bar_peer": list(self.bar.peer_ptrs), "ctl": self.ctl.data_ptr()}

    def check(self, what: str = "distributed GEMM") -> None:
        self.status.check(what)


class ShardedRows:
    """bf16 ``[R*S, cols]`` in symmetric memory; group member q owns rows ``[q*S, (q+1)*S)``."""

    def __init__(self, ctx: DistGemmContext, group: list[int], rows_per_rank: int, cols: int, *,
                 chunk_rows: int | None = None, ld: int | None = None):
        self.ctx, self.group = ctx, list(group)
        self.R = len(group)
        self.my = self.group.index(ctx.rank)
        self.S, self.cols = int(rows_per_rank), int(cols)
        self.ld = int(ld or _round_up(cols, 8))
        if chunk_rows is None:
            chunk_rows = next(c for c in (128, 64, 32, 16, 8, 4, 2, 1) if self.S % c == 0)
        if self.S % chunk_rows:
            raise ValueError("chunk_rows must divide the rows per rank")
        self.chunk_rows = int(chunk_rows)
        self.buf = ctx.heap.alloc((self.R * self.S, self.ld), torch.bfloat16)
        self.buf.local.zero_()
        self.ready = torch.zeros(self.R * self.S // self.chunk_rows, dtype=torch.int32, device=ctx.device)
        self.done = torch.zeros_like(self.ready)

    @property
    def full(self) -> torch.Tensor:
        """All rows (valid after a gathering GEMM ran), padded pitch."""
        return self.buf.local

    @property
    def local(self) -> torch.Tensor:
        """This rank's rows (padded pitch)."""
        return self.buf.local[self.my * self.S:(self.my + 1) * self.S]

    def gather_spec(self) -> dict | None:
        if self.R == 1:
            return None
        pieces, per = _pieces(self.chunk_rows, self.cols)
        return {"nranks": self.R, "my": self.my, "src": [self.buf.peer_ptrs[g] for g in self.group],
                "dst": self.buf.local.data_ptr(), "ld": self.ld, "rows_per_rank": self.S,
                "row_elems": _round_up(self.cols, 8), "chunk_rows": self.chunk_rows,
                "pieces": pieces, "piece_vecs": per, "ready": self.ready.data_ptr(), "done": self.done.data_ptr()}

    def column_view(self, col_offset: int, cols: int) -> "ShardedRowsView":
        """The columns [col_offset, col_offset+cols) as a separately gatherable operand."""
        return ShardedRowsView(self, col_offset, cols)


class ShardedRowsView:
    """A column range of a ``ShardedRows`` buffer with its own ready flags."""

    def __init__(self, base: ShardedRows, col_offset: int, cols: int):
        if col_offset % 8 or col_offset + cols > base.ld:
            raise ValueError("column views start at a multiple of 8 elements and stay inside the row")
        self.base, self.off, self.cols = base, int(col_offset), int(cols)
        self.R, self.my, self.S, self.ld, self.group = base.R, base.my, base.S, base.ld, base.group
        self.chunk_rows = base.chunk_rows
        self.ready = torch.zeros_like(base.ready)
        self.done = torch.zeros_like(base.ready)

    @property
    def full(self) -> torch.Tensor:
        return self.base.buf.local[:, self.off:self.off + self.cols]

    @property
    def local(self) -> torch.Tensor:
        return self.base.buf.local[self.my * self.S:(self.my + 1) * self.S, self.off:self.off + self.cols]

    def gather_spec(self) -> dict | None:
        if self.R == 1:
            return None
        return {"nranks": self.R, "my": self.my, "src": [p + 2 * self.off for p in
                                                         (self.base.buf.peer_ptrs[g] for g in self.group)],
                "dst": self.base.buf.local.data_ptr() + 2 * self.off, "ld": self.ld, "rows_per_rank": self.S,
                "row_elems": _round_up(self.cols, 8), "chunk_rows": self.chunk_rows,
                "pieces": _pieces(self.chunk_rows, self.cols)[0], "piece_vecs": _pieces(self.chunk_rows, self.cols)[1],
                "ready": self.ready.data_ptr(), "done": self.done.data_ptr()}


class RowReduceScatter:
    """Receive blocks (bf16, one 32 x 32 block per sender/tile/quarter/column chunk) and
    per-(tile, lane quarter, column half) flags for a row reduce-scatter."""

    def __init__(self, ctx: DistGemmContext, group: list[int], rows_per_rank: int, max_cols: int):
        if rows_per_rank % BM:
            raise ValueError("reduce-scatter rows per rank must be a multiple of 128")
        self.ctx, self.group = ctx, list(group)
        self.R = len(group)
        self.my = self.group.index(ctx.rank)
        self.S = int(rows_per_rank)
        self.ld = _round_up(max_cols, 8)
        self.max_cols = int(max_cols)
        self.recv = ctx.heap.alloc((self.R, self.S, _round_up(max_cols, BN)), torch.bfloat16)
        tiles_per_rank = (self.S // BM) * ((max_cols + BN - 1) // BN)
        self.flags = ctx.heap.alloc((self.R * tiles_per_rank * 8,), torch.int32)
        self.flags.local.zero_()

    def spec(self, n_cols: int) -> dict | None:
        if self.R == 1:
            return None
        if n_cols > self.max_cols:
            raise ValueError("reduce-scatter output wider than its buffers")
        return {"nranks": self.R, "my": self.my, "rows_per_rank": self.S,
                "recv_peer": [self.recv.peer_ptrs[g] for g in self.group], "recv_local": self.recv.local.data_ptr(),
                "flag_peer": [self.flags.peer_ptrs[g] for g in self.group],
                "flag_local": self.flags.local.data_ptr()}


def tile_order(M: int, N: int, *, ga: dict | None = None, gb: dict | None = None, rs: dict | None = None,
               a_mn: bool = False, b_mn: bool = False) -> list[int]:
    """Processing order of the output tiles: ready data first, sends before own rows."""
    mt_n, nt_n = (M + BM - 1) // BM, (N + BN - 1) // BN

    def dist(row: int, g: dict) -> int:
        return ((row // g["rows_per_rank"]) - g["my"]) % g["nranks"]

    keys = []
    for mt in range(mt_n):
        for nt in range(nt_n):
            da = dist(mt * BM, ga) if ga is not None and not a_mn else 0
            db = dist(nt * BN, gb) if gb is not None and not b_mn else 0
            if rs is not None:
                owner = (mt * BM) // rs["rows_per_rank"]
                own = 1 if owner == rs["my"] else 0
                key = (own, (owner - rs["my"]) % rs["nranks"], db, mt, nt)
            else:
                key = (max(da, db), da + db, mt, nt)
            keys.append((key, (mt << 16) | nt))
    keys.sort()
    return [k[1] for k in keys]


def chunk_order(ga: dict | None, gb: dict | None) -> list[int]:
    """Copy work items (``operand << 31 | chunk << 12 | piece``) of the remote chunks:
    nearest owner first, operands interleaved, a chunk's pieces consecutive (so the
    copy warps of many CTAs finish each chunk together)."""
    out = []
    rmax = max(g["nranks"] for g in (ga, gb) if g is not None) if (ga or gb) else 1
    for d in range(1, rmax):
        for op, g in ((0, ga), (1, gb)):
            if g is None or d >= g["nranks"]:
                continue
            owner = (g["my"] + d) % g["nranks"]
            per = g["rows_per_rank"] // g["chunk_rows"]
            pieces = g.get("pieces", 1)
            for c in range(owner * per, (owner + 1) * per):
                out.extend(((op << 31) | (c << 12) | k) - (1 << 32 if op else 0) for k in range(pieces))
    return out


def _mat(t: torch.Tensor, transposed: bool) -> tuple[int, int, int]:
    if t.dim() != 2 or t.stride(1) != 1 or t.dtype != torch.bfloat16:
        raise ValueError("distributed GEMM operands must be 2-D bf16 with unit inner stride")
    return (t.shape[1], t.shape[0], t.stride(0)) if transposed else (t.shape[0], t.shape[1], t.stride(0))


@dataclass
class DistGemm:
    """One bound call site: ``out = epi(A @ B^T)`` with optional fused gathers / reduce-scatter.

    ``a``/``b`` are the logical operands (for a gathered operand: the FULL
    buffer ``ShardedRows.full`` sliced to the used columns); ``a_t``/``b_t``
    mean the stored matrix is the transpose.  With ``rs`` the output ``out``
    holds this rank's rows only.
    """

    ctx: DistGemmContext
    a: torch.Tensor
    b: torch.Tensor
    out: torch.Tensor
    a_t: bool = False
    b_t: bool = False
    ga: "ShardedRows | ShardedRowsView | None" = None
    gb: "ShardedRows | ShardedRowsView | None" = None
    rs: RowReduceScatter | None = None
    bias: torch.Tensor | None = None
    relu: bool = False
    mask: torch.Tensor | None = None
    colsum: torch.Tensor | None = None
    alpha: float = 1.0
    accumulate: bool = False
    epi: str = "plain"
    aux0: torch.Tensor | None = None
    aux1: torch.Tensor | None = None
    zout: torch.Tensor | None = None

    def __post_init__(self):
        M, K, lda = _mat(self.a, self.a_t)
        N, Kb, ldb = _mat(self.b, self.b_t)
        if K != Kb:
            raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
        out = self.out
        if out.dtype not in (torch.float32, torch.bfloat16) or out.stride(1) != 1:
            raise ValueError("output must be fp32/bf16 with unit inner stride")
        ga = self.ga.gather_spec() if self.ga is not None else None
        gb = self.gb.gather_spec() if self.gb is not None else None
        rs = self.rs.spec(N) if self.rs is not None else None
        rows_out = M // self.rs.R if self.rs is not None else M
        if out.shape[0] < rows_out or out.shape[1] < N:
            raise ValueError("output too small")
        tiles = tile_order(M, N, ga=ga, gb=gb, rs=rs, a_mn=self.a_t, b_mn=self.b_t)
        chunks = chunk_order(ga, gb)
        dev = out.device
        self._tiles = torch.tensor(tiles, dtype=torch.int32, device=dev)
        self._chunks = torch.tensor(chunks or [0], dtype=torch.int32, device=dev)
        epi = {"plain": 0, "cross": 1, "residual": 2}[self.epi]
        g = {"A": self.a.data_ptr(), "lda": lda, "a_mn": self.a_t, "B": self.b.data_ptr(), "ldb": ldb,
             "b_mn": self.b_t, "M": M, "N": N, "K": K, "C": out.data_ptr(), "ldc": out.stride(0),
             "c_dtype": F32 if out.dtype == torch.float32 else BF16, "accumulate": self.accumulate,
             "bias": self.bias.data_ptr() if self.bias is not None else 0, "act": 1 if self.relu else 0,
             "alpha": float(self.alpha), "mask": self.mask.data_ptr() if self.mask is not None else 0,
             "ldm": self.mask.stride(0) if self.mask is not None else 0,
             "colsum": self.colsum.data_ptr() if self.colsum is not None else 0,
             "status": self.ctx.status.ptr, "timeout_ns": self.ctx.timeout_ns}
        d = {"g": g, "tiles": self._tiles.data_ptr(), "num_tiles": len(tiles), "chunks": self._chunks.data_ptr(),
             "num_chunks": len(chunks), "ga": ga, "gb": gb, "rs": rs, "epi": epi, **self.ctx.fields()}
        for name, t in (("aux0", self.aux0), ("aux1", self.aux1), ("zout", self.zout)):
            if t is not None:
                d[name] = t.data_ptr()
                d["ld" + ("0" if name == "aux0" else "1" if name == "aux1" else "z")] = t.stride(0)
        self._d = d
        self.M, self.N, self.K = M, N, K

    def __call__(self) -> torch.Tensor:
        native().gemm_dist(self._d)
        return self.out

    @property
    def flops(self) -> int:
        return 2 * self.M * self.N * self.K


__all__ = ["DistGemm", "DistGemmContext", "RowReduceScatter", "ShardedRows", "ShardedRowsView", "chunk_order",
           "tile_order"]
