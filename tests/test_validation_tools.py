"""Validation tools: Perfetto timeline round trip, phase overlap, reader interleave and locality (CPU)."""
import json

import pytest

from flare_b200.validation.overlap import effective_overlap, phase_overlap
from flare_b200.validation.perfetto import PerfettoWriter, parse_trace, step_statistics
from flare_b200.validation.readers import (read_position_audit, validate_interleave_restore,
                                           validate_reader_locality)


def test_perfetto_round_trip(tmp_path):
    w = PerfettoWriter()
    w.slice(("rank:0", "compute"), "train_core", 1_000, 5_000, step=3, loss=0.25, tag="a", neg=-7, ok=True)
    w.slice(("rank:1", "data"), "prepare_bind", 2_000, 2_500, step=4)
    w.instant(("rank:0", "compute"), "marker", 4_000, note="x")
    ev = parse_trace(w.save(tmp_path / "t.pftrace"))
    by = {e["name"]: e for e in ev}
    t = by["train_core"]
    assert (t["ts_ns"], t["dur_ns"], t["track"]) == (1_000, 4_000, "rank:0/compute")
    assert t["payload"] == {"step": 3, "loss": 0.25, "tag": "a", "neg": -7, "ok": True}
    assert by["prepare_bind"]["track"] == "rank:1/data" and by["marker"]["dur_ns"] == 0
    st = step_statistics(ev, name="train_core", global_batch_size=1000)
    assert st["count"] == 1 and st["max_ms"] == pytest.approx(0.004)


def _timeline(tmp_path):
    w = PerfettoWriter()
    for step in range(4):
        t0 = 10_000_000 * step
        w.slice(("rank:0", "compute"), "train_core", t0, t0 + 8_000_000, step=step)
        # the next step's inputs are materialised while this step trains: fully hidden
        w.slice(("rank:0", "data"), "prepare_sparse_materialize", t0 + 1_000_000, t0 + 3_000_000, step=step + 1)
        # the previous step's scatter: half before this step's end, half after
        w.slice(("rank:0", "data"), "scatter_sparse_grads", t0 + 7_000_000, t0 + 9_000_000, step=step - 1)
    return parse_trace(w.save(tmp_path / "tl.pftrace"))


def test_phase_overlap_and_effective_summary(tmp_path):
    rep = phase_overlap(_timeline(tmp_path), {1, 2})
    rows = {r["step"]: r for r in rep["rows"]}
    mat = rows[1]["overlaps"]["materialize_next"]
    assert mat["present"] and mat["hidden_ms"] == pytest.approx(2.0) and mat["hidden_fraction_of_candidate"] == 1.0
    sc = rows[2]["overlaps"]["scatter_prev"]
    assert sc["hidden_ms"] == pytest.approx(1.0) and sc["overlap_ms"] == pytest.approx(1.0)
    eff = effective_overlap(rep, min_hidden_fraction=0.5)
    assert eff["relations"]["materialize_next"]["total_hidden_fraction"] == pytest.approx(1.0)
    assert eff["overlap_proven"]
    strict = effective_overlap(rep, min_hidden_fraction=0.9)
    assert "scatter_prev" in strict["blockers"] and not strict["overlap_proven"]


def test_reader_interleave_across_a_restore(tmp_path):
    pa = pytest.importorskip("pyarrow")
    pq = pytest.importorskip("pyarrow.parquet")
    from flare_b200.data.reader import BatchReader
    from flare_b200.data.sources import ParquetSourceFactory

    paths = []
    for f in range(4):
        p = tmp_path / f"f{f}.parquet"
        pq.write_table(pa.table({"x": list(range(f * 1000, f * 1000 + 120))}), p, row_group_size=30)
        paths.append(str(p))
    fac = ParquetSourceFactory(paths)
    first, states = [], []
    for r in range(2):
        rd = BatchReader(fac, 10, rank=r, world=2, position_audit_path=tmp_path / f"a{r}.jsonl")
        it = iter(rd)
        for _ in range(4):
            next(it)
        states.append(rd.capture_state())
        rd.close()
        first += (tmp_path / f"a{r}.jsonl").read_text().splitlines()
    second = []
    for r in range(3):
        rd = BatchReader(fac, 10, rank=r, world=3, position_audit_path=tmp_path / f"b{r}.jsonl")
        rd.restore_state(states)
        it = iter(rd)
        for _ in range(3):
            next(it)
        rd.close()
        second += (tmp_path / f"b{r}.jsonl").read_text().splitlines()
    res = validate_interleave_restore(read_position_audit(first, 2), read_position_audit(second, 3), initial_world=2,
                                      restored_world=3, initial_steps=8, restored_steps=9)
    assert res["exact"] and res["topology"] == "2->3"
    with pytest.raises(AssertionError):
        validate_interleave_restore(read_position_audit(first, 2), read_position_audit(second, 3), initial_world=2,
                                    restored_world=3, initial_steps=8, restored_steps=10)
    with pytest.raises(ValueError):
        read_position_audit(first + first[:1], 2)  # a position read twice


def test_reader_locality_against_placement():
    from flare_b200.runtime.placement import (DEFAULT_ROLE_PROFILES, NodeSpec, ResourceProfiles,
                                              resolve_resource_profiles, solve_placement)

    nodes = [NodeSpec("hostA", 64, 2, 512e9), NodeSpec("hostB", 64, 2, 512e9)]
    counts = {"rank": 4, "reader": 8}
    prof = resolve_resource_profiles(counts) if callable(resolve_resource_profiles) else ResourceProfiles(
        DEFAULT_ROLE_PROFILES)
    pl = solve_placement(nodes, counts, prof)
    hosts = [nodes[n].name for n in pl.rank_node]
    out = validate_reader_locality(pl, hosts, minimum_nodes=2)
    assert len(out["lanes"]) == 8 and out["nodes"] == ["hostA", "hostB"]
    with pytest.raises(ValueError):
        validate_reader_locality(pl, list(reversed(hosts)))
    pl.reader_node[0] = 1 - pl.reader_node[0]  # a lane moved off its rank's node
    with pytest.raises(ValueError):
        validate_reader_locality(pl, hosts)
