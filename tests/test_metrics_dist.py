"""Exact metric merges over gloo ranks: the partitioned merge (groups and score ranges split over the
ranks) equals the all-gather merge and the one-process oracle, with ties across ranks, groups split
over ranks, a rank with no samples and several world sizes (CPU)."""
import numpy as np
import pytest
import torch

from flare_b200.metrics.ranking import auc_reference, gauc_reference
from flare_b200.testing.gloo import run_ranks


def _data(n=4000, seed=3):
    rng = np.random.default_rng(seed)
    s = (rng.integers(0, 200, n) / 200).astype(np.float32)  # heavy ties
    y = (rng.random(n) < 0.25 + 0.5 * s).astype(np.float32)
    g = rng.integers(0, 97, n).astype(np.int64)
    return s, y, g


def _worker(rank, world, empty_rank):
    from flare_b200.metrics.distributed import distributed_metrics

    s, y, g = _data()
    idx = np.arange(len(s))
    mine = idx[idx % world == rank] if rank != empty_rank else idx[:0]
    if empty_rank >= 0 and rank == (empty_rank + 1) % world:  # the empty rank's share goes to its neighbour
        mine = np.concatenate([mine, idx[idx % world == empty_rank]])
    ts, ty, tg = (torch.from_numpy(a[mine]) for a in (s, y, g))
    part = distributed_metrics(ts, ty, tg, negative_factor=0.5, merge="partitioned")
    full = distributed_metrics(ts, ty, tg, negative_factor=0.5, merge="allgather")
    return part, full


@pytest.mark.parametrize("world,empty_rank", [(2, -1), (3, 1), (4, -1)])
def test_partitioned_merge_is_exact(world, empty_rank):
    s, y, g = _data()
    want_auc, want_gauc = auc_reference(s, y), gauc_reference(s, y, g, 0.5)
    for part, full in run_ranks(_worker, world, empty_rank):
        assert abs(part["auc"] - want_auc) < 1e-12 and abs(full["auc"] - want_auc) < 1e-12
        assert abs(part["gauc"] - want_gauc) < 1e-12 and abs(full["gauc"] - want_gauc) < 1e-12
        assert abs(part["calibration"] - full["calibration"]) < 1e-12


def test_unknown_merge_is_rejected():
    from flare_b200.metrics.distributed import distributed_metrics

    with pytest.raises(ValueError, match="merge"):
        distributed_metrics(torch.rand(4), torch.ones(4), merge="tree")
