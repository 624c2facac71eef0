"""Mesh layout and DCN config arithmetic (CPU)."""
import pytest

from flare_b200.models.dcn import DCNConfig, dcn_benchmark_tables
from flare_b200.parallel.mesh import DeviceMesh2D, SparsePartitionMapping


def test_mesh_groups_tp_innermost():
    m = DeviceMesh2D(2, 4)
    assert m.world == 8
    assert m.tp_group(5) == [4, 5]
    assert m.fsdp_group(5) == [1, 3, 5, 7]
    assert m.coords(6) == (0, 3)
    assert DeviceMesh2D.for_world(1, 2) == DeviceMesh2D(1, 1)
    with pytest.raises(ValueError):
        DeviceMesh2D.for_world(3, 2)
    for r in range(8):
        assert r in m.tp_group(r) and r in m.fsdp_group(r)
        assert set(m.tp_group(r)) & set(m.fsdp_group(r)) == {r}


def test_sparse_partition_mapping_is_independent_of_dense_mesh():
    sp = SparsePartitionMapping.over_node(8)
    assert sp.num_partitions == 8 and sp.partition_of(3) == 3


def test_dcn_config_widths_and_flops():
    cfg = DCNConfig(tables=dcn_benchmark_tables([1000] * 26, 256))
    assert cfg.width == 6669
    W = 6669
    expect = 3 * (3 * 2 * 2 * W * 512 + 2 * (W * 4096 + 3 * 4096 * 4096) + 2 * (W + 4096))
    assert cfg.dense_flops_per_sample() == expect
    with pytest.raises(ValueError):
        DCNConfig(tables=dcn_benchmark_tables([10] * 2, 64), deep=(256, 256, 256), tp=2)
