"""Elastic restart on CPU gloo ranks: a rank fails (host-side exception) mid-run; the job restarts at
another world size from the last committed checkpoint and ends in exactly the state of a run that
changed world size at that checkpoint without failing."""
import torch

from flare_b200.recipes.cpu_elastic import elastic_cpu_worker
from flare_b200.runtime.elastic import run_elastic
from flare_b200.runtime.launch import spawn_ranks


def _same(a, b):
    if isinstance(a, dict):
        assert set(a) == set(b)
        for k in a:
            _same(a[k], b[k])
    elif isinstance(a, (list, tuple)):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            _same(x, y)
    elif torch.is_tensor(a):
        assert torch.equal(a, b)
    else:
        assert a == b


def test_elastic_restart_resumes_from_the_last_committed_checkpoint(tmp_path):
    G, seed, every = 64, 0, 2
    # reference: 2 ranks for steps 1-4 (checkpoints at 2 and 4), then 1 rank from step 4 to 8
    ref = tmp_path / "ref"
    spawn_ranks(elastic_cpu_worker, 2, str(ref), 4, G, seed, every, None)
    want = spawn_ranks(elastic_cpu_worker, 1, str(ref), 8, G, seed, every, None)[0]
    assert want["start"] == 4

    # elastic: rank 1 of 2 fails before step 6 (steps 5 is lost: after the last checkpoint)
    res = run_elastic(elastic_cpu_worker, [2, 1], str(tmp_path / "el"), 8, G, seed, every, (1, 6), max_restarts=2,
                      pg_timeout_s=8.0)
    assert [a.ok for a in res.attempts] == [False, True] and [a.world for a in res.attempts] == [2, 1]
    got = res.results[0]
    assert got["start"] == 4 and sorted(got["losses"]) == [5, 6, 7, 8]
    committed = sorted(p.name for p in (tmp_path / "el" / "steps").iterdir() if not p.name.endswith(".partial"))
    assert committed == ["2", "4", "6", "8"]
    _same(got["losses"], want["losses"])
    _same(got["sparse"]["tables"], want["sparse"]["tables"])
    _same(got["dense"], want["dense"])


def test_a_rank_that_exits_without_a_result_is_a_rank_failure():
    import pytest

    from flare_b200.runtime.launch import RankFailure
    from flare_b200.testing.gloo import exit_silently_worker

    with pytest.raises(RankFailure) as e:
        spawn_ranks(exit_silently_worker, 2, timeout=60.0)
    assert e.value.rank == 1 and "exited with code 3" in e.value.detail and set(e.value.failed) == {1}


def test_elastic_restart_after_a_silent_exit():
    from flare_b200.testing.gloo import exit_silently_worker

    res = run_elastic(exit_silently_worker, [2, 1], max_restarts=1, timeout=60.0)
    assert [a.ok for a in res.attempts] == [False, True] and res.attempts[0].failed_rank == 1
    assert res.results == [0]
