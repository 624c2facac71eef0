"""Host-tier directory: residency, CLOCK victims and the two-step protection window (CPU)."""
import numpy as np
import pytest

from flare_b200.sparse.host_tier import HostShard


def _shard(rows, C):
    hs = object.__new__(HostShard)
    hs.rows, hs.C = rows, C
    hs.slot_of = np.full(rows, -1, dtype=np.int32)
    hs.row_of = np.full(C, -1, dtype=np.int64)
    hs.stamp = np.full(C, -(1 << 40), dtype=np.int64)
    hs.hand = 0
    hs.stats = {"hits": 0, "misses": 0, "evictions": 0}
    return hs


def test_plan_keeps_directory_consistent_and_protects_recent_steps():
    rng = np.random.default_rng(0)
    hs = _shard(5000, 600)
    prev = np.zeros(0, np.int64)
    for step in range(1, 40):
        rows = np.unique(rng.integers(0, 5000, 250))
        p = hs.plan(step, rows)
        # every row of the step is resident afterwards, in a slot that maps back to it
        assert (hs.slot_of[rows] >= 0).all()
        assert (hs.row_of[hs.slot_of[rows]] == rows).all()
        # victims never come from the previous step or this step
        assert not np.isin(p.evict_rows, prev).any() and not np.isin(p.evict_rows, rows).any()
        assert len(set(p.miss_slots.tolist())) == len(p.miss_slots)
        res = np.nonzero(hs.row_of >= 0)[0]
        assert (hs.slot_of[hs.row_of[res]] == res).all()
        assert int((hs.slot_of >= 0).sum()) == len(res)
        prev = rows
    assert hs.stats["evictions"] > 0


def test_cache_too_small_for_two_steps_raises():
    hs = _shard(1000, 100)
    hs.plan(1, np.arange(60))
    with pytest.raises(RuntimeError):
        hs.plan(2, np.arange(100, 160))
