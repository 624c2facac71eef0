"""Hash-keyed tables on the CPU collection: insert on first sight, LFU eviction, eval lookups (CPU)."""
import pytest
import torch

from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.reference import CpuEmbeddingBagCollection


def _batch(keys_per_sample):
    lens = torch.tensor([len(k) for k in keys_per_sample])
    offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).int()
    vals = torch.tensor([k for ks in keys_per_sample for k in ks], dtype=torch.int32)
    return offs, vals


@pytest.mark.parametrize("native", [False, True])
def test_dynamic_table_lookup_insert_and_lfu_eviction(native):
    opt = SparseOptimizerConfig(kind="sgd", learning_rate=0.5)
    t = SparseTableSpec("users", 4, 8, dynamic=True, optimizer=opt)
    c = CpuEmbeddingBagCollection([t], 3, optimizer=opt, native=native)
    offs, vals = _batch([[1_000_003], [7, 1_000_003], [42]])
    c.set_input(offs, vals)
    y = c.forward()
    keys, slots, uses = c.dynamic_items(0)
    row = dict(zip(keys.tolist(), slots.tolist()))
    assert set(row) == {1_000_003, 7, 42} and dict(zip(keys.tolist(), uses.tolist()))[1_000_003] == 2
    w = c.weights[0]
    torch.testing.assert_close(y[0], w[row[1_000_003]])
    torch.testing.assert_close(y[1], w[row[7]] + w[row[1_000_003]])
    before = w.clone()
    c.backward(torch.ones_like(y))
    assert torch.equal(w[row[42]], before[row[42]] - 0.5)  # plain SGD on the rows the batch touched

    # capacity 4: 3 used; two new keys -> one free slot + evict the least used key not in this batch
    offs, vals = _batch([[5], [6], [1_000_003]])
    c.set_input(offs, vals)
    c.forward()
    keys = set(c.dynamic_items(0)[0].tolist())
    assert keys == {5, 6, 1_000_003, 7} or keys == {5, 6, 1_000_003, 42}
    evicted = ({7, 42} - keys).pop()
    # eval lookups insert nothing: an unknown (evicted) key pools to zero
    offs, vals = _batch([[evicted], [5], []])
    c.set_input(offs, vals)
    y = c.forward(training=False)
    assert torch.count_nonzero(y[0]) == 0 and torch.count_nonzero(y[2]) == 0 and torch.count_nonzero(y[1]) > 0
    assert set(c.dynamic_items(0)[0].tolist()) == keys


def test_dynamic_table_overflow_is_reported():
    t = SparseTableSpec("items", 2, 4, dynamic=True)
    c = CpuEmbeddingBagCollection([t], 1)
    offs, vals = _batch([[1, 2, 3]])
    c.set_input(offs, vals)
    with pytest.raises(RuntimeError, match="dynamic table full"):
        c.forward()


def test_dynamic_table_on_paged_storage(tmp_path):
    from flare_b200.sparse.storage import SparseStorageOptions

    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.1)
    t = SparseTableSpec("u", 5000, 8, dynamic=True, optimizer=opt)
    c = CpuEmbeddingBagCollection([t], 2, optimizer=opt, storage=SparseStorageOptions(
        memory_limit_bytes=4096 * 9 * 4, spill_directory=str(tmp_path), entries_per_page=4096))
    offs, vals = _batch([[123456789, 5], [5]])
    c.set_input(offs, vals)
    y = c.forward()
    c.backward(torch.ones_like(y))
    keys, slots, uses = c.dynamic_items(0)
    assert sorted(keys.tolist()) == [5, 123456789] and sorted(uses.tolist()) == [1, 2]
    assert y.abs().max() <= 2 * t.init_scale + 1e-6


@pytest.mark.parametrize("paged", [False, True])
def test_cpu_collection_state_round_trip_resumes_identically(tmp_path, paged):
    from flare_b200.sparse.storage import SparseStorageOptions

    opt = SparseOptimizerConfig(kind="adam", learning_rate=0.05)
    # 8 slots for 12 distinct keys: the resumed run must evict exactly as the original
    tables = [SparseTableSpec("d", 8, 8, dynamic=True, optimizer=opt), SparseTableSpec("s", 50, 4, optimizer=opt)]
    B = 4
    mk = lambda: CpuEmbeddingBagCollection(  # noqa: E731
        tables, B, optimizer=opt, seed=2,
        storage=SparseStorageOptions(memory_limit_bytes=4096 * 64, spill_directory=str(tmp_path)) if paged else None)
    g = torch.Generator().manual_seed(0)

    def batch():
        lens = torch.randint(1, 3, (2 * B,), generator=g)
        offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).int()
        vals = torch.cat([torch.randint(0, 10**9, (int(lens[:B].sum()),), generator=g) % 12 * 7919,
                          torch.randint(0, 50, (int(lens[B:].sum()),), generator=g)]).int()
        return offs, vals

    def step(c, b):
        c.set_input(*b)
        y = c.forward()
        c.backward(torch.cos(y))
        return y

    a = mk()
    for _ in range(3):
        step(a, batch())
    state = a.state_dict()
    b = mk()
    b.load_state_dict(state)
    for _ in range(3):
        nb = batch()
        torch.testing.assert_close(step(b, nb), step(a, nb), rtol=0, atol=0)
    assert b.state_dict()["step"] == a.state_dict()["step"] == 6
