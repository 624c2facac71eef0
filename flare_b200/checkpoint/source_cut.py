"""The input cut of a checkpoint: every reader's position, committed with the model state.

A training checkpoint restores exactly only if the input resumes where the saved model stopped.
``save_reader_cut`` writes one rank's reader state (``data.reader.BatchReader.capture_state``: the
items it fully consumed, the row offset inside the current one, its position counters) into
``steps/<step>[.partial]/reader/rank<k>.json`` beside the model and sparse parts, so it is committed
by the same rename; ``load_reader_cut`` returns every saved rank's state for
``BatchReader.restore_state``, which deals the remaining items to any number of new ranks.

``inspect_source_cut`` is the offline consistency check of one committed step: the step directory is
committed (not ``.partial``); there is one reader file per rank of the saving run, each naming this
step, its own rank and the same world size (``expected_readers`` when given); no item is consumed by
two ranks and no rank's partly read item is another rank's consumed one.  It returns a summary: the
readers, the items consumed, the global input positions consumed (base + every rank's batches) and
the partly read items.  It checks the files' agreement with each other and with the step, not that a
restart after a crash replays nothing twice (that needs an interrupted run).

    python -m flare_b200.checkpoint.source_cut CKPT_ROOT STEP [--expected-readers N]

Reference behaviour: the reader's cut-position checkpoint (src/flare/runtime/fluxway/workers/
reader.py:396-416) committed with the model state, and the source-cut inspection of
tools/validation/inspect_checkpoint_source_cut.py.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
from typing import Any

from ..io.artifacts import write_json
from .store import step_dir

FORMAT = "flare_b200.reader_cut.v1"


def _reader_dir(dirpath: str | os.PathLike) -> Path:
    return Path(dirpath) / "reader"


def save_reader_cut(dirpath: str | os.PathLike, step: int, state: dict[str, Any]) -> Path:
    """Write one rank's reader ``state`` into the step directory ``dirpath`` (usually the ``.partial``
    one, before the commit)."""
    for key in ("rank", "world", "done"):
        if key not in state:
            raise ValueError(f"reader state lacks {key!r}")
    d = _reader_dir(dirpath)
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"rank{int(state['rank'])}.json"
    write_json(path, {"format": FORMAT, "step": int(step), "state": state})
    return path


def load_reader_cut(dirpath: str | os.PathLike) -> list[dict[str, Any]]:
    """Every saved rank's reader state of a step directory, in rank order ([] when none were saved)."""
    d = _reader_dir(dirpath)
    if not d.is_dir():
        return []
    out = []
    for p in sorted(d.glob("rank*.json"), key=lambda q: int(q.stem[4:])):
        rec = json.loads(p.read_text())
        if rec.get("format") != FORMAT:
            raise ValueError(f"{p}: not a reader cut file")
        out.append(rec["state"])
    return out


def inspect_source_cut(root: str | os.PathLike, step: int, expected_readers: int | None = None) -> dict[str, Any]:
    """Check that step ``step``'s reader cut is complete and self-consistent; raise ``AssertionError`` if not."""
    if step < 0:
        raise ValueError("step must be non-negative")
    d = step_dir(root, step)
    if not d.is_dir():
        partial = d.with_name(f"{d.name}.partial")
        raise AssertionError(f"step {step} is not committed" + (" (only a .partial directory)" if partial.exists()
                                                                 else ""))
    files = sorted(_reader_dir(d).glob("rank*.json"), key=lambda q: int(q.stem[4:]))
    if not files:
        raise AssertionError(f"step {step} has no reader cut")
    recs = [json.loads(p.read_text()) for p in files]
    for p, rec in zip(files, recs):
        if rec.get("format") != FORMAT:
            raise AssertionError(f"{p.name}: unknown format {rec.get('format')!r}")
        if rec.get("step") != step:
            raise AssertionError(f"{p.name}: cut of step {rec.get('step')!r}, checkpoint step {step}")
        if int(rec["state"]["rank"]) != int(p.stem[4:]):
            raise AssertionError(f"{p.name}: holds the state of rank {rec['state']['rank']}")
    worlds = {int(rec["state"]["world"]) for rec in recs}
    if len(worlds) != 1:
        raise AssertionError(f"reader files disagree on the world size: {sorted(worlds)}")
    world = worlds.pop()
    if expected_readers is not None and world != expected_readers:
        raise AssertionError(f"saved by {world} readers, expected {expected_readers}")
    ranks = sorted(int(rec["state"]["rank"]) for rec in recs)
    if ranks != list(range(world)):
        raise AssertionError(f"reader files of ranks {ranks}, expected ranks 0..{world - 1}")
    owner: dict[int, int] = {}
    for rec in recs:
        r = int(rec["state"]["rank"])
        for item in rec["state"]["done"]:
            if item in owner:
                raise AssertionError(f"item {item} consumed by ranks {owner[item]} and {r}")
            owner[item] = r
    partial = {}
    for rec in recs:
        cur = rec["state"].get("current")
        if cur:
            item, row = int(cur[0]), int(cur[1])
            if item in owner:
                raise AssertionError(f"item {item} is partly read by rank {rec['state']['rank']} but consumed by "
                                     f"rank {owner[item]}")
            partial[item] = row
    base = max(int(rec["state"].get("position_base", 0)) for rec in recs)
    positions = base + sum(int(rec["state"].get("batches", 0)) for rec in recs)
    return {"step": step, "readers": world, "items_consumed": len(owner), "positions_consumed": positions,
            "partial_items": {str(k): v for k, v in sorted(partial.items())}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="offline consistency check of a checkpoint's reader cut")
    ap.add_argument("root")
    ap.add_argument("step", type=int)
    ap.add_argument("--expected-readers", type=int, default=None)
    args = ap.parse_args(argv)
    if args.expected_readers is not None and args.expected_readers <= 0:
        raise SystemExit("--expected-readers must be positive")
    out = inspect_source_cut(args.root, args.step, args.expected_readers)
    print("checkpoint_source_cut_consistent=true")
    for k, v in out.items():
        print(f"checkpoint_{k}={json.dumps(v) if isinstance(v, dict) else v}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["FORMAT", "inspect_source_cut", "load_reader_cut", "save_reader_cut"]
