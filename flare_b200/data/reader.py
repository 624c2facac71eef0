"""Per-rank batch reader: assigned work items, resumable cut position, audit, global valid count.

``BatchReader`` reads the work items of a ``SourceFactory`` assigned to this
rank (item k goes to rank ``k % world``), cuts them into fixed-size batches
under a completion policy and yields ``(batch, validity)``.  Its checkpoint
state is the cut position only: the global ids of the items fully consumed
and the row offset inside the current one.  ``restore_state`` accepts a
state saved at any world size (global reshard): the union of every rank's
saved states marks the consumed items, and the remaining items are dealt to
the new ranks.  ``repeat_first_batch`` replays the first batch forever (the
simulation mode used to measure the training path without input cost).
``close`` writes an audit JSON (items, rows, batches, padded rows, errors,
seconds).  ``global_valid_count`` sums the valid samples of a step over the
ranks and checks it against the scheduled work.

Reference behaviour: src/flare/runtime/fluxway/workers/reader.py:77-516
(BatchReaderSPMD: assigned reads, repeat-first-batch, capture / restore of
the cut position, audit at shutdown) and recipes/recsys/ranking/workers/
reader.py:148-166 (global valid-prefix count).
"""
from __future__ import annotations

import time
from collections.abc import Callable, Iterator
from pathlib import Path
from typing import Any

from ..io.artifacts import write_json
from .sources import BatchAssembler, SourceFactory, WorkItem


class BatchReader:
    def __init__(self, factory: SourceFactory, batch_size: int, *, rank: int = 0, world: int = 1,
                 policy: str = "pad", repeat_first_batch: bool = False, audit_path: str | Path | None = None,
                 transform: Callable[[Any], Any] | None = None, position_audit_path: str | Path | None = None):
        if not 0 <= rank < world:
            raise ValueError("rank must be in [0, world)")
        self.factory, self.B, self.rank, self.world = factory, int(batch_size), rank, world
        self.policy, self.repeat = policy, bool(repeat_first_batch)
        self.audit_path = Path(audit_path) if audit_path else None
        self.transform = transform or (lambda x: x)
        self.items: list[WorkItem] = [it for it in factory.plan() if it.item_id % world == rank]
        self.done: set[int] = set()        # global ids of fully consumed items
        self.cur_item: int | None = None   # global id of the item being read
        self.cur_row = 0                   # rows of it already handed out
        self.stats = {"items": 0, "rows": 0, "batches": 0, "padded_rows": 0, "errors": 0}
        self._t0 = time.time()
        # global step positions: the readers interleave (position p is read by rank p % world), so
        # this rank's k-th batch since the last restore is the k-th position at or after the base
        # that is congruent to its rank (one JSON line each in the position audit)
        self.position_base = 0
        self.position_audit_path = Path(position_audit_path) if position_audit_path else None
        self.positions: list[dict] = []

    # ------------------------------------------------------------------ state
    def capture_state(self) -> dict:
        return {"rank": self.rank, "world": self.world, "done": sorted(self.done),
                "current": None if self.cur_item is None else [self.cur_item, self.cur_row],
                "position_base": self.position_base, "batches": len(self.positions)}

    def restore_state(self, states: list[dict]) -> None:
        """Resume from the saved states of every rank of the previous run (any world size)."""
        done: set[int] = set()
        partial: dict[int, int] = {}
        for st in states:
            done.update(st["done"])
            if st.get("current"):
                item, row = st["current"]
                partial[item] = max(partial.get(item, 0), row)
        self.done = done
        # positions consumed by the saved run: its base plus every rank's batches since then
        self.position_base = max((int(st.get("position_base", 0)) for st in states), default=0) + \
            sum(int(st.get("batches", 0)) for st in states)
        self.positions = []
        all_items = [it for it in self.factory.plan() if it.item_id not in done]
        self.items = [it for k, it in enumerate(all_items) if k % self.world == self.rank]
        self._partial = {k: v for k, v in partial.items() if k not in done}

    # ------------------------------------------------------------------ reading
    def _chunks(self) -> Iterator[tuple[int, Any, int, int]]:
        session = self.factory.create_session()
        partial = getattr(self, "_partial", {})
        try:
            for it in self.items:
                if it.item_id in self.done:
                    continue
                table = session.read(it)
                skip = partial.get(it.item_id, 0)
                rows = table.num_rows if hasattr(table, "num_rows") else len(next(iter(table.values())))
                if skip:
                    table = table.slice(skip) if hasattr(table, "slice") else {k: v[skip:] for k, v in table.items()}
                yield it.item_id, table, rows - skip, skip
        finally:
            session.close()

    def _advance(self, valid: int) -> None:
        """Account ``valid`` more rows handed out: items whose rows are all out are done."""
        self._emitted += valid
        while self._pushed and self._pushed[0][2] <= self._emitted:
            self.done.add(self._pushed.pop(0)[0])
            self.stats["items"] += 1
        if self._pushed and self._pushed[0][1] < self._emitted:
            item, start, _, skip = self._pushed[0]
            self.cur_item, self.cur_row = item, skip + self._emitted - start
        else:
            self.cur_item, self.cur_row = None, 0

    def __iter__(self):
        asm = BatchAssembler(self.B, self.policy)
        self._pushed: list[tuple[int, int, int, int]] = []  # (item, first row, end row, skipped rows)
        self._emitted, pushed_rows, first = 0, 0, None
        for item, table, n, skip in self._chunks():
            self._pushed.append((item, pushed_rows, pushed_rows + n, skip))
            pushed_rows += n
            self.stats["rows"] += n
            if n == 0:
                self._advance(0)
            for ab in asm.push(table):
                if self.repeat:
                    first = first or ab
                    while True:
                        self.stats["batches"] += 1
                        self._note_position()
                        yield self.transform(first.data), first.validity
                self.stats["batches"] += 1
                self._advance(ab.validity.valid_count)
                self._note_position()
                yield self.transform(ab.data), ab.validity
        for ab in asm.finish():
            self.stats["batches"] += 1
            self.stats["padded_rows"] += ab.validity.batch_size - ab.validity.valid_count
            self._advance(ab.validity.valid_count)
            self._note_position()
            yield self.transform(ab.data), ab.validity
        # rows the completion policy dropped at the end of the stream are consumed too
        self._advance(pushed_rows - self._emitted)

    def _note_position(self) -> None:
        k = len(self.positions)
        first = self.position_base + (self.rank - self.position_base) % self.world
        self.positions.append({"position": first + k * self.world, "rank": self.rank,
                               "world_size": self.world})

    # ------------------------------------------------------------------ accounting
    def close(self) -> dict:
        audit = {**self.stats, "rank": self.rank, "world": self.world, "seconds": time.time() - self._t0,
                 "assigned_items": [it.item_id for it in self.items], "done": sorted(self.done)}
        if self.audit_path is not None:
            write_json(self.audit_path, audit)
        if self.position_audit_path is not None:
            import json

            self.position_audit_path.write_text("".join(json.dumps(p) + "\n" for p in self.positions))
        return audit


def reconcile_reader_audits(audits: list[dict], planned_items: list[int] | None = None,
                            planned_rows: int | None = None) -> dict:
    """Check the readers' audits of one run against each other and against the plan.

    Every planned item must be consumed by exactly one rank (``done`` of its
    audit), no rank may report an item outside the plan, and the rows the
    ranks read must add up to ``planned_rows`` when given.  Returns a report
    with ``ok`` and the offending item ids.  Reference behaviour: the reader
    audit reconciliation tool of tools/validation (reader execution audits
    written at shutdown, src/flare/runtime/fluxway/workers/reader.py:455-477).
    """
    owner: dict[int, list[int]] = {}
    for a in audits:
        for item in a.get("done", []):
            owner.setdefault(int(item), []).append(int(a.get("rank", -1)))
    duplicated = sorted(i for i, rs in owner.items() if len(rs) > 1)
    planned = set(planned_items) if planned_items is not None else None
    missing = sorted(planned - owner.keys()) if planned is not None else []
    unexpected = sorted(owner.keys() - planned) if planned is not None else []
    rows = sum(int(a.get("rows", 0)) for a in audits)
    errors = sum(int(a.get("errors", 0)) for a in audits)
    rows_ok = planned_rows is None or rows == planned_rows
    ranks = sorted(int(a.get("rank", -1)) for a in audits)
    worlds = {int(a.get("world", len(audits))) for a in audits}
    ranks_ok = len(worlds) == 1 and ranks == list(range(worlds.pop()))
    return {"ok": not duplicated and not missing and not unexpected and rows_ok and ranks_ok and errors == 0,
            "items_consumed": len(owner), "duplicated": duplicated, "missing": missing, "unexpected": unexpected,
            "rows": rows, "planned_rows": planned_rows, "errors": errors, "ranks": ranks, "ranks_complete": ranks_ok,
            "padded_rows": sum(int(a.get("padded_rows", 0)) for a in audits),
            "seconds_max": max((float(a.get("seconds", 0.0)) for a in audits), default=0.0)}


def global_valid_count(valid: int, *, expected: int | None = None) -> int:
    """Valid samples of this step summed over the ranks (int32 all-reduce); checked against ``expected``."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([int(valid)], dtype=torch.int32)
    if dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() == "nccl":
            t = t.cuda()
        dist.all_reduce(t)
    total = int(t.item())
    if expected is not None and total != expected:
        raise RuntimeError(f"global valid samples {total} differ from the scheduled {expected}")
    return total


def main(argv=None) -> int:
    """``python -m flare_b200.data.reader AUDIT.json... [--items N] [--rows R]``: reconcile audits (exit 1 if not ok)."""
    import argparse
    import json

    p = argparse.ArgumentParser(prog="flare_b200.data.reader")
    p.add_argument("audits", nargs="+")
    p.add_argument("--items", type=int, default=None, help="planned item count (ids 0..N-1)")
    p.add_argument("--rows", type=int, default=None, help="planned row count")
    args = p.parse_args(argv)
    audits = [json.loads(Path(f).read_text()) for f in args.audits]
    rep = reconcile_reader_audits(audits, list(range(args.items)) if args.items is not None else None, args.rows)
    print(json.dumps(rep, indent=1))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["BatchReader", "global_valid_count", "reconcile_reader_audits"]
