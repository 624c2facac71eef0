"""Checks of the input readers: step interleave across a restore, reader-to-rank locality.

* ``validate_interleave_restore``: the readers of a run deal global step
  positions round-robin (position p is read by rank ``p % world``).  Given
  the position audits (``BatchReader(position_audit_path=...)``, one JSON line
  ``{"position", "rank", "world_size"}`` per batch) of a run and of its
  continuation restored at another world size, check that each run covers
  exactly its positions with the right ranks and that the continuation
  starts where the first run stopped.
* ``validate_reader_locality``: every reader lane of a placement
  (``runtime.placement.solve_placement``) must run on the node of the rank
  it feeds, and the planned nodes must be the nodes the processes report at
  run time (``attest_nodes``: every rank's host name, gathered over the
  process group).

    python -m flare_b200.validation.readers interleave first.jsonl second.jsonl \\
        --initial-world-size 2 --restored-world-size 3 --initial-steps 8 --restored-steps 9

Reference counterparts: tools/validation/validate_interleave_restore.py and
tools/validation/validate_reader_locality.py.
"""
from __future__ import annotations

import argparse
import json
import socket
from pathlib import Path
from typing import Any


def read_position_audit(lines, world_size: int) -> dict[int, int]:
    """position -> rank from audit lines (or a path); each position must appear once."""
    if isinstance(lines, (str, Path)):
        lines = Path(lines).read_text().splitlines()
    seen: dict[int, int] = {}
    for n, line in enumerate(lines, 1):
        if not str(line).strip():
            continue
        ev = json.loads(line) if isinstance(line, str) else dict(line)
        if set(ev) != {"position", "rank", "world_size"}:
            raise ValueError(f"line {n}: not a reader position event: {ev}")
        if int(ev["world_size"]) != world_size:
            raise ValueError(f"line {n}: world size {ev['world_size']}, expected {world_size}")
        p = int(ev["position"])
        if p in seen:
            raise ValueError(f"position {p} read twice")
        seen[p] = int(ev["rank"])
    return seen


def validate_interleave_restore(initial: dict[int, int], restored: dict[int, int], *, initial_world: int,
                                restored_world: int, initial_steps: int, restored_steps: int) -> dict[str, Any]:
    for name, v in (("initial_world", initial_world), ("restored_world", restored_world),
                    ("initial_steps", initial_steps), ("restored_steps", restored_steps)):
        if v <= 0:
            raise ValueError(f"{name} must be positive")
    want_a = {p: p % initial_world for p in range(initial_steps)}
    want_b = {p: p % restored_world for p in range(initial_steps, initial_steps + restored_steps)}
    if initial != want_a:
        missing = sorted(set(want_a) - set(initial))[:8]
        raise AssertionError(f"first run's interleave differs (missing {missing}, "
                             f"wrong ranks {[p for p in initial if want_a.get(p) != initial[p]][:8]})")
    if restored != want_b:
        missing = sorted(set(want_b) - set(restored))[:8]
        raise AssertionError(f"restored run's interleave differs (missing {missing}, "
                             f"wrong ranks {[p for p in restored if want_b.get(p) != restored[p]][:8]})")
    return {"topology": f"{initial_world}->{restored_world}", "positions": initial_steps + restored_steps,
            "exact": True}


def attest_nodes() -> list[str]:
    """Every rank's host name, in rank order (one all-gather; this rank only without a process group)."""
    import torch.distributed as dist

    me = socket.gethostname()
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [me]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, me)
    return list(out)


def validate_reader_locality(placement, attested_rank_hosts: list[str], *, minimum_nodes: int = 1) -> dict[str, Any]:
    """``placement``: a ``runtime.placement.Placement``; ``attested_rank_hosts``: host of every rank at run time."""
    names = [n.name for n in placement.nodes]
    ranks = len(placement.rank_node)
    if len(attested_rank_hosts) != ranks:
        raise ValueError(f"{len(attested_rank_hosts)} attested ranks, the placement has {ranks}")
    for r, node in enumerate(placement.rank_node):
        if names[node] != attested_rank_hosts[r]:
            raise ValueError(f"rank {r} was placed on {names[node]} but runs on {attested_rank_hosts[r]}")
    if len(set(attested_rank_hosts)) < minimum_nodes:
        raise ValueError(f"the ranks span {len(set(attested_rank_hosts))} nodes, fewer than {minimum_nodes}")
    lanes = []
    for lane, (node, rank) in enumerate(zip(placement.reader_node, placement.reader_rank)):
        if node != placement.rank_node[rank]:
            raise ValueError(f"reader lane {lane} runs on {names[node]} but feeds rank {rank} on "
                             f"{names[placement.rank_node[rank]]}")
        lanes.append({"lane": lane, "rank": rank, "node": names[node]})
    return {"evidence": "placement reader lanes and run-time host names", "nodes": sorted(set(attested_rank_hosts)),
            "lanes": lanes}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("interleave")
    a.add_argument("initial_audit")
    a.add_argument("restored_audit")
    for k in ("initial-world-size", "restored-world-size", "initial-steps", "restored-steps"):
        a.add_argument(f"--{k}", type=int, required=True)
    args = ap.parse_args(argv)
    res = validate_interleave_restore(read_position_audit(args.initial_audit, args.initial_world_size),
                                      read_position_audit(args.restored_audit, args.restored_world_size),
                                      initial_world=args.initial_world_size, restored_world=args.restored_world_size,
                                      initial_steps=args.initial_steps, restored_steps=args.restored_steps)
    print(json.dumps(res))


if __name__ == "__main__":
    main()


__all__ = ["attest_nodes", "read_position_audit", "validate_interleave_restore", "validate_reader_locality"]
