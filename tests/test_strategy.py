"""Named-axis rank mesh and sharding strategies (CPU): coordinates, groups, shard specs, ZeRO stage
partitions, checkpoint sharding on the first divisible dimension, and shard / assemble round trips."""
import pytest
import torch

from flare_b200.parallel.mesh import DeviceMesh2D
from flare_b200.parallel.strategy import (CheckpointShardingStrategy, DataParallelStrategy, ParallelMesh,
                                          ZeroShardingStrategy)
from flare_b200.training.contracts import TrainingExecutionPlan, ZeroStage


def test_mesh_coordinates_and_groups_match_the_2d_layout():
    m = ParallelMesh.from_axes(fsdp=4, tp=2)
    d2 = DeviceMesh2D(tp=2, fsdp=4)
    assert m.size == 8 and m.axis_size("tp") == 2
    for r in range(8):
        c = m.coords(r)
        assert (c["tp"], c["fsdp"]) == d2.coords(r) and m.rank_of(**c) == r
        assert m.group("tp", r) == d2.tp_group(r)
        assert m.group("fsdp", r) == d2.fsdp_group(r)
    assert m.groups("tp") == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert m.group(("fsdp", "tp"), 5) == list(range(8))
    with pytest.raises(ValueError, match="not present"):
        m.axis_size("dp")
    with pytest.raises(ValueError, match="does not match"):
        ParallelMesh.from_axes(world_size=6, fsdp=4, tp=2)
    with pytest.raises(ValueError, match="unique"):
        ParallelMesh(("a", "a"), (1, 2))


def test_shard_and_assemble_round_trip():
    m = ParallelMesh.from_axes(fsdp=2, tp=2)
    x = torch.arange(8 * 6, dtype=torch.float32).view(8, 6)
    spec = m.named("fsdp", "tp")
    shards = {r: m.shard(x, spec, r) for r in range(4)}
    assert shards[1].shape == (4, 3) and torch.equal(shards[1], x[0:4, 3:6])
    assert torch.equal(m.assemble(shards, spec, (8, 6)), x)
    both = m.named(("fsdp", "tp"))
    assert torch.equal(m.shard(x, both, 3), x[6:8])
    with pytest.raises(ValueError, match="divide"):
        m.local_slice(m.named("tp"), (5,), 0)
    with pytest.raises(ValueError, match="cover"):
        m.assemble({0: shards[0]}, spec, (8, 6))


def test_data_parallel_and_zero_partitions():
    m = ParallelMesh.from_dp(4, axis_name="fsdp")
    dp = DataParallelStrategy(m, "fsdp")
    assert dp.batch_sharding().dims == ("fsdp",) and dp.replicated.is_replicated
    specs = {s: ZeroShardingStrategy(m, s) for s in ZeroStage}
    assert specs[ZeroStage.REPLICATED].zero_optimizer_sharding().is_replicated
    assert not specs[ZeroStage.OPTIMIZER_STATE].zero_optimizer_sharding().is_replicated
    assert specs[ZeroStage.OPTIMIZER_STATE].zero_gradient_sharding().is_replicated
    assert not specs[ZeroStage.GRADIENT].zero_gradient_sharding().is_replicated
    assert specs[ZeroStage.GRADIENT].zero_parameter_sharding().is_replicated
    assert not specs[ZeroStage.PARAMETER].zero_parameter_sharding().is_replicated
    z = specs[ZeroStage.OPTIMIZER_STATE]
    st = z.zero_state_specs(2, 5)
    assert [s.is_replicated for s in st] == [True, True, False, False, False]
    assert len(z.zero_gradient_specs(3)) == 3
    with pytest.raises(ValueError):
        z.zero_state_specs(4, 3)
    # flattened state split in equal padded blocks
    lin = torch.nn.Linear(3, 3)  # 9 weights padded to 12 -> four blocks of 3
    blocks = [ZeroShardingStrategy(m, ZeroStage.PARAMETER).shard_model(lin, r)["weight"] for r in range(4)]
    assert [b.numel() for b in blocks] == [3, 3, 3, 3]
    assert torch.equal(torch.cat(blocks)[:9], lin.weight.detach().reshape(-1)) and not blocks[3].any()
    plan = TrainingExecutionPlan.sharded(ZeroStage.GRADIENT)
    zs = ZeroShardingStrategy.from_execution_plan(plan, ParallelMesh.from_dp(2, axis_name=plan.zero.axis_name))
    assert zs.stage == ZeroStage.GRADIENT


def test_checkpoint_sharding_first_divisible_dimension():
    m = ParallelMesh.from_axes(node=2, fsdp=4)
    cs = CheckpointShardingStrategy(m, "fsdp")
    assert cs.checkpoint_sharding((6, 8)).dims == (None, "fsdp")
    assert cs.checkpoint_sharding((12, 8)).dims == ("fsdp",)
    assert cs.checkpoint_sharding((3, 5)).is_replicated
    assert CheckpointShardingStrategy(ParallelMesh.from_axes(fsdp=1), "fsdp").checkpoint_sharding((8,)).is_replicated
    state = {"w": torch.randn(6, 8), "b": torch.randn(3), "e": torch.randn(16, 2)}
    per_rank = {r: cs.local_shards(state, r) for r in range(8)}
    assert "b" in per_rank[0] and "b" not in per_rank[1] and per_rank[1]["w"].shape == (6, 2)
    back = cs.assemble({r: per_rank[r] for r in range(4)}, {k: tuple(v.shape) for k, v in state.items()})
    for k in state:
        assert torch.equal(back[k], state[k])
