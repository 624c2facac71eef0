"""Table-wise sharded CPU collection over gloo ranks equals one collection on the global batch (CPU)."""
import pytest
import torch

from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.testing.gloo import run_ranks

OPT = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.1)
TABLES = [SparseTableSpec(f"t{i}", n, d, optimizer=OPT, pooling="mean" if i == 1 else "sum")
          for i, (n, d) in enumerate([(50, 8), (30, 4), (70, 8), (20, 12), (40, 4)])]
B = 6


def _global_batch(step, world):
    g = torch.Generator().manual_seed(100 + step)
    GB = B * world
    lens = torch.randint(0, 4, (len(TABLES), GB), generator=g)
    ids = [torch.randint(0, t.num_embeddings, (int(lens[f].sum()),), generator=g) for f, t in enumerate(TABLES)]
    return lens, ids


def _local(lens, ids, rank, bsz):
    """Rank's KJT: its ``bsz`` samples of every feature."""
    vals, ls = [], []
    for f in range(len(TABLES)):
        cum = torch.cat([torch.zeros(1, dtype=torch.long), lens[f].cumsum(0)])
        lo, hi = int(cum[rank * bsz]), int(cum[(rank + 1) * bsz])
        vals.append(ids[f][lo:hi])
        ls.append(lens[f][rank * bsz:(rank + 1) * bsz])
    ls = torch.cat(ls)
    offs = torch.cat([torch.zeros(1, dtype=torch.long), ls.cumsum(0)]).int()
    return offs, torch.cat(vals).int()


def _run(rank, world, native, steps=3):
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    c = ShardedCpuEmbeddingBagCollection(TABLES, B, optimizer=OPT, seed=7, native=native)
    outs = []
    for s in range(steps):
        lens, ids = _global_batch(s, world)
        c.set_input(*_local(lens, ids, rank, B))
        y = c.forward()
        outs.append(y)
        c.backward(torch.tanh(y) * 0.5)  # per-sample gradients: rows of the global batch's gradient
    return outs, {f: c.table_weights(f) for f in range(len(TABLES)) if c.table_weights(f) is not None}


@pytest.mark.parametrize("native", [False, True])
def test_two_ranks_equal_one_collection_on_the_global_batch(native):
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    ref = ShardedCpuEmbeddingBagCollection(TABLES, 2 * B, optimizer=OPT, seed=7, native=native)  # world 1
    ref_outs = []
    for s in range(3):
        lens, ids = _global_batch(s, 2)
        ref.set_input(*_local(lens, ids, 0, 2 * B))
        y = ref.forward()
        ref_outs.append(y)
        ref.backward(torch.tanh(y) * 0.5)
    results = run_ranks(_run, 2, native)
    for r, (outs, tabs) in enumerate(results):
        for s in range(3):
            torch.testing.assert_close(outs[s], ref_outs[s][r * B:(r + 1) * B], rtol=0, atol=0)
        for f, w in tabs.items():
            assert f % 2 == r  # table-wise placement
            torch.testing.assert_close(w, ref.table_weights(f), rtol=0, atol=0)
    assert sorted(f for _, tabs in results for f in tabs) == list(range(len(TABLES)))


def _recipe(rank, world):
    from flare_b200.recipes.cpu_small import train_small_cpu

    return train_small_cpu(steps=8, batch_size=16).losses


def test_cpu_recipe_over_two_gloo_ranks_tracks_one_rank():
    from flare_b200.recipes.cpu_small import train_small_cpu

    one = train_small_cpu(steps=8, batch_size=32).losses
    two = run_ranks(_recipe, 2)
    assert two[0] == two[1]  # the global-mean loss is the same on every rank
    for a, b in zip(one, two[0]):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (one, two[0])


def _train_and_save(rank, world):
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    c = ShardedCpuEmbeddingBagCollection(TABLES, B, optimizer=OPT, seed=7)
    for s in range(2):
        lens, ids = _global_batch(s, world)
        c.set_input(*_local(lens, ids, rank, B))
        y = c.forward()
        c.backward(torch.tanh(y) * 0.5)
    return c.state_dict()


def test_sharded_state_restores_at_another_world_size():
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    states = run_ranks(_train_and_save, 2)  # 2 ranks, each with its own tables
    assert sorted(n for st in states for n in st["tables"]) == sorted(t.name for t in TABLES)
    ref = ShardedCpuEmbeddingBagCollection(TABLES, 2 * B, optimizer=OPT, seed=7)  # one rank, straight through
    resumed = ShardedCpuEmbeddingBagCollection(TABLES, 2 * B, optimizer=OPT, seed=0)
    resumed.load_state_dict(states)  # one rank restored from the two ranks' states
    for s in range(4):
        lens, ids = _global_batch(s, 2)
        for c in ([ref] if s < 2 else [ref, resumed]):
            c.set_input(*_local(lens, ids, 0, 2 * B))
            y = c.forward()
            c.backward(torch.tanh(y) * 0.5)
    for f in range(len(TABLES)):
        torch.testing.assert_close(resumed.table_weights(f), ref.table_weights(f), rtol=0, atol=0)


DYN_TABLES = [SparseTableSpec("d0", 64, 8, optimizer=OPT, dynamic=True),
              SparseTableSpec("s1", 30, 4, optimizer=OPT),
              SparseTableSpec("d2", 48, 4, optimizer=OPT, dynamic=True)]


def _dyn_batch(step, world):
    """Keys of the dynamic tables widen with the step: later steps insert keys never seen before."""
    g = torch.Generator().manual_seed(300 + step)
    GB = B * world
    lens = torch.randint(1, 4, (len(DYN_TABLES), GB), generator=g)
    ids = []
    for f, t in enumerate(DYN_TABLES):
        hi = 1000 * (f + 1) + 5 * (step + 1) if t.dynamic else t.num_embeddings
        lo = 1000 * (f + 1) if t.dynamic else 0
        ids.append(torch.randint(lo, hi, (int(lens[f].sum()),), generator=g))
    return lens, ids


def _dyn_local(lens, ids, rank, bsz):
    vals, ls = [], []
    for f in range(len(DYN_TABLES)):
        cum = torch.cat([torch.zeros(1, dtype=torch.long), lens[f].cumsum(0)])
        lo, hi = int(cum[rank * bsz]), int(cum[(rank + 1) * bsz])
        vals.append(ids[f][lo:hi])
        ls.append(lens[f][rank * bsz:(rank + 1) * bsz])
    ls = torch.cat(ls)
    return torch.cat([torch.zeros(1, dtype=torch.long), ls.cumsum(0)]).int(), torch.cat(vals).int()


def _dyn_steps(c, rank, world, bsz, steps):
    for s in steps:
        lens, ids = _dyn_batch(s, world)
        c.set_input(*_dyn_local(lens, ids, rank, bsz))
        y = c.forward()
        c.backward(torch.tanh(y) * 0.5)


def _dyn_train_save(rank, world):
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    c = ShardedCpuEmbeddingBagCollection(DYN_TABLES, B, optimizer=OPT, seed=7)
    _dyn_steps(c, rank, world, B, range(2))
    return c.state_dict()


def _dyn_resume_two(rank, world, states):
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    c = ShardedCpuEmbeddingBagCollection(DYN_TABLES, B, optimizer=OPT, seed=123)  # the state brings the streams
    c.load_state_dict(states)
    _dyn_steps(c, rank, world, B, range(2, 5))
    return {f: c.table_weights(f) for f in range(len(DYN_TABLES)) if c.table_weights(f) is not None}


def test_dynamic_tables_resume_bitwise_with_new_keys_after_the_restore():
    """Hash-keyed tables keep inserting keys after a restore; their new rows come from each table's
    own init stream, carried in the checkpoint, so a resumed run matches the straight-through run
    bitwise at the same world size and at another one."""
    from flare_b200.sparse.cpu_sharded import ShardedCpuEmbeddingBagCollection

    states = run_ranks(_dyn_train_save, 2)
    ref = ShardedCpuEmbeddingBagCollection(DYN_TABLES, 2 * B, optimizer=OPT, seed=7)
    _dyn_steps(ref, 0, 2, 2 * B, range(5))
    one = ShardedCpuEmbeddingBagCollection(DYN_TABLES, 2 * B, optimizer=OPT, seed=0)
    one.load_state_dict(states)
    _dyn_steps(one, 0, 2, 2 * B, range(2, 5))
    two = run_ranks(_dyn_resume_two, 2, states)
    merged = {f: w for part in two for f, w in part.items()}
    for f in range(len(DYN_TABLES)):
        torch.testing.assert_close(one.table_weights(f), ref.table_weights(f), rtol=0, atol=0)
        torch.testing.assert_close(merged[f], ref.table_weights(f), rtol=0, atol=0)
