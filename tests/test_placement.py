"""Role profiles and rank placement (CPU)."""
import pytest

from flare_b200.runtime.placement import (GiB, NodeSpec, ResourceProfile, resolve_resource_profiles,
                                          solve_placement)


def test_resolve_profiles_validation_and_overrides():
    p = resolve_resource_profiles({"rank": 8, "reader": 16})
    assert p.get_role("rank").demand()["GPU"] == 1
    cpu = resolve_resource_profiles({"rank": 2}, compute_device="cpu")
    assert cpu.get_role("rank").demand()["GPU"] == 0
    with pytest.raises(ValueError):
        resolve_resource_profiles({"rank": 0})
    with pytest.raises(KeyError):
        resolve_resource_profiles({"rank": 1, "mystery": 1})
    with pytest.raises(KeyError):
        p.get_role("metrics")
    with pytest.raises(ValueError):
        ResourceProfile(base={"CPU": 1}).demand(3) if False else p.get_role("rank").demand(10**6)


def test_two_nodes_tp_groups_and_reader_colocation():
    nodes = [NodeSpec("a", 112, 8, 1500 * GiB), NodeSpec("b", 112, 8, 1500 * GiB)]
    prof = resolve_resource_profiles({"rank": 16, "reader": 32, "metrics": 2})
    pl = solve_placement(nodes, {"rank": 16, "reader": 32, "metrics": 2}, prof, tp=2)
    assert pl.rank_node == [0] * 8 + [1] * 8
    assert all(pl.reader_node[l] == pl.rank_node[pl.reader_rank[l]] for l in range(32))
    assert pl.local_ranks()[8:] == list(range(8))
    assert sorted(pl.role_nodes["metrics"]) == [0, 1]
    assert pl.launch_plan()["b"][0] == (8, 0)
    # balanced growth: every rank gets the same number of scale steps on identical nodes
    assert max(pl.scale_steps) - min(pl.scale_steps) <= 1 and min(pl.scale_steps) > 0
    for u, n in zip(pl.usage, nodes):
        assert u["memory"] <= n.memory and u["CPU"] <= n.cpus


def test_capacity_and_straddle_errors():
    prof = resolve_resource_profiles({"rank": 6})
    with pytest.raises(ValueError):
        solve_placement([NodeSpec("a", 64, 4, 512 * GiB)], {"rank": 6}, prof)
    two = [NodeSpec("a", 64, 6, 512 * GiB), NodeSpec("b", 64, 6, 512 * GiB)]
    with pytest.raises(ValueError):  # 8 ranks do not form groups of 3
        solve_placement(two, {"rank": 8}, resolve_resource_profiles({"rank": 8}), tp=3)
    # groups of 4 on 6-GPU nodes: a node takes whole groups only
    pl = solve_placement(two, {"rank": 8}, resolve_resource_profiles({"rank": 8}), tp=4)
    assert pl.rank_node == [0] * 4 + [1] * 4
    with pytest.raises(ValueError):
        solve_placement([NodeSpec("a", 8, 8, 512 * GiB)], {"rank": 8}, resolve_resource_profiles({"rank": 8}))
    with pytest.raises(ValueError):
        solve_placement([NodeSpec("a", 64, 8, 1024 * GiB)], {"rank": 8}, resolve_resource_profiles({"rank": 8}),
                        policy="feasible", target_scale_steps=200)
