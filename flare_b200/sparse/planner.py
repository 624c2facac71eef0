"""Embedding sharding planner: table-wise, column-wise and row-wise placement.

A rank holds whole tables (table-wise), column slices of tables
(column-wise), or row-wise pieces: a table with ``shards = R > 1`` is cut by
key modulo R, piece r holding rows ``i % R == r`` (the reference's modulo
key partitioning, src/flare/runtime/fluxway/workers/dynamic_embedding.py:
43-66, src/flare/mesh/topology.py:20-35).  Table-wise and column-wise
shards produce complete columns of the pooled output, so no partial sums
cross NVLink; row-wise pieces produce fp32 partial sums that the requester
adds in residue order.  Row-wise pieces spread a table too large for one
GPU (or too hot for one) over several, and every row keeps its optimizer
state in one place, so row-wise optimizers stay exact.

Placement balances lookup work (``expected lookups x columns``, divided by R
for a row-wise piece) with a longest-processing-time greedy pass, splitting
the heaviest whole-row piece on the most loaded rank in half (by columns)
while that lowers the maximum load, subject to an HBM budget per rank.
"""
from __future__ import annotations

from dataclasses import dataclass

from .config import SparseTableSpec

VALID_SHARD_WIDTHS = (4, 8, 16, 32, 64, 128, 256)


@dataclass(frozen=True)
class ShardPlacement:
    table: int      # index into the table list
    col_begin: int
    ncols: int
    rank: int
    row_index: int = 0    # row-wise piece: holds table rows i with i % row_shards == row_index
    row_shards: int = 1

    def num_rows(self, num_embeddings: int) -> int:
        return (num_embeddings - self.row_index + self.row_shards - 1) // self.row_shards


@dataclass(frozen=True)
class ShardingPlan:
    world_size: int
    placements: tuple[ShardPlacement, ...]
    out_cols: tuple[int, ...]   # pooled-output column of each table's first column
    total_dim: int

    def for_rank(self, rank: int) -> list[ShardPlacement]:
        return [p for p in self.placements if p.rank == rank]

    def load(self, work) -> list[float]:
        loads = [0.0] * self.world_size
        for p in self.placements:
            loads[p.rank] += work[p.table] * p.ncols / p.row_shards
        return loads

    def row_shards(self, table: int) -> int:
        return max([p.row_shards for p in self.placements if p.table == table], default=1)


def _bytes_per_elem(dtype: str) -> int:
    return 4 if dtype == "float32" else 2


def plan_sharding(
    tables: list[SparseTableSpec],
    world_size: int,
    *,
    expected_lookups: list[float] | None = None,
    hbm_budget_bytes: float | None = None,
    max_rounds: int = 64,
    allow_rowwise_column_split: bool = False,
    row_split: bool = True,
    rw_overhead: float = 0.06,
) -> ShardingPlan:
    """Place tables (or column slices, or row-wise pieces) on ranks.

    Column splits are made only for tables whose optimizer is elementwise:
    a row-wise optimizer (row-wise Adagrad/Adam) keeps one state value per
    row, and splitting columns would give each slice its own state, which
    changes the update.  ``allow_rowwise_column_split`` permits it anyway
    (per-slice row state, as some embedding libraries do).  Where a column
    split is not allowed, ``row_split`` lets the balancing rounds double a
    table's row-wise pieces instead (exact for every optimizer); each piece
    is charged ``rw_overhead`` of the table's work for its partial-sum rows
    and its pull of the pooled gradients.  ``expected_lookups`` is the
    relative work per column of each table (lookups, plus the unique rows the
    backward updates: ``estimate_table_costs``).
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    for t in tables:
        if t.embedding_dim not in VALID_SHARD_WIDTHS:
            raise ValueError(f"table {t.name}: embedding_dim must be one of {VALID_SHARD_WIDTHS}")
    work = list(expected_lookups) if expected_lookups is not None else [1.0] * len(tables)
    out_cols, c = [], 0
    for t in tables:
        out_cols.append(c)
        c += t.embedding_dim
    # pieces: (table, col_begin, ncols, row_index, row_shards)
    pieces = []
    for i, t in enumerate(tables):
        R = max(1, int(t.shards))
        pieces += [(i, 0, t.embedding_dim, r, R) for r in range(R)]

    def pwork(pc):
        return work[pc[0]] * pc[2] * (1.0 / pc[4] + (rw_overhead if pc[4] > 1 else 0.0))

    def assign(pcs):
        order = sorted(range(len(pcs)), key=lambda k: (-pwork(pcs[k]), pcs[k][0], pcs[k][3], pcs[k][1]))
        loads = [0.0] * world_size
        mem = [0.0] * world_size
        owner = [0] * len(pcs)
        for k in order:
            ti, _, nc, _, R = pcs[k]
            nbytes = tables[ti].num_embeddings / R * nc * _bytes_per_elem(tables[ti].value_dtype)
            cands = sorted(range(world_size), key=lambda r: (loads[r], mem[r], r))
            chosen = cands[0]
            if hbm_budget_bytes is not None:
                fits = [r for r in cands if mem[r] + nbytes <= hbm_budget_bytes]
                if not fits:
                    raise MemoryError(f"table {tables[ti].name} piece does not fit the HBM budget on any rank")
                chosen = fits[0]
            owner[k] = chosen
            loads[chosen] += pwork(pcs[k])
            mem[chosen] += nbytes
        return owner, loads

    owner, loads = assign(pieces)

    def score(ld):
        top = max(ld)
        return (round(top, 6), sum(1 for x in ld if abs(x - top) < 1e-9))

    if world_size > 1:
        best = (score(loads), pieces, owner, loads)
        for _ in range(max_rounds):
            hot = loads.index(max(loads))
            cand = [k for k in range(len(pieces)) if owner[k] == hot and pieces[k][2] // 2 in VALID_SHARD_WIDTHS
                    and pieces[k][2] >= 32 and pieces[k][4] == 1
                    and (allow_rowwise_column_split or not tables[pieces[k][0]].optimizer.needs_row_state)]
            if cand:
                k = max(cand, key=lambda k: (pwork(pieces[k]), -k))
                ti, cb, nc, _, _ = pieces[k]
                pieces = pieces[:k] + [(ti, cb, nc // 2, 0, 1), (ti, cb + nc // 2, nc // 2, 0, 1)] + pieces[k + 1:]
            else:
                # double the row-wise pieces of the heaviest full-width table on the hot rank
                rcand = [k for k in range(len(pieces)) if owner[k] == hot and row_split
                         and pieces[k][2] == tables[pieces[k][0]].embedding_dim
                         and pieces[k][4] * 2 <= world_size and not tables[pieces[k][0]].dynamic
                         and tables[pieces[k][0]].cache_rows is None
                         and tables[pieces[k][0]].num_embeddings >= 2 * pieces[k][4]]
                if not rcand:
                    break
                ti = pieces[max(rcand, key=lambda k: (pwork(pieces[k]), -k))][0]
                R = next(pc[4] for pc in pieces if pc[0] == ti) * 2
                dim = tables[ti].embedding_dim
                pieces = [pc for pc in pieces if pc[0] != ti] + [(ti, 0, dim, r, R) for r in range(R)]
            owner, loads = assign(pieces)
            if score(loads) < best[0]:
                best = (score(loads), pieces, owner, loads)
        _, pieces, owner, loads = best
    placements = tuple(ShardPlacement(ti, cb, nc, owner[k], r, R) for k, (ti, cb, nc, r, R) in enumerate(pieces))
    return ShardingPlan(world_size, placements, tuple(out_cols), c)


def estimate_table_costs(vocab_sizes: list[int], lookups: int, zipf_s: float = 1.05, *, unique_weight: float = 2.0,
                         seed: int = 0, device="cpu") -> list[float]:
    """Relative per-column work of each table for ``lookups`` Zipf(``zipf_s``) ids per step.

    Work = lookups (forward gather, backward gradient gather) + ``unique_weight`` x the
    distinct rows a step touches (the backward reads and writes each once), counted on a
    sample of the id distribution, normalised by ``lookups``.
    """
    import torch

    from ..data.synthetic import zipf_ids

    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for v in vocab_sizes:
        u = torch.unique(zipf_ids(int(lookups), int(v), zipf_s, g, device=device)).numel()
        out.append(1.0 + unique_weight * u / float(lookups))
    return out


__all__ = ["ShardPlacement", "ShardingPlan", "VALID_SHARD_WIDTHS", "estimate_table_costs", "plan_sharding"]
