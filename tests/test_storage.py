"""Paged row store with a memory limit and disk spill, and the CPU collection on top of it."""
import pytest
import torch

from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.reference import CpuEmbeddingBagCollection
from flare_b200.sparse.storage import SparseStorageOptions


def test_options_validation(tmp_path):
    with pytest.raises(ValueError, match="entries_per_page"):
        SparseStorageOptions(entries_per_page=1000)
    with pytest.raises(ValueError, match="spill directory"):
        SparseStorageOptions(max_spill_bytes=1 << 20)
    with pytest.raises(ValueError, match="positive"):
        SparseStorageOptions(memory_limit_bytes=0, spill_directory=str(tmp_path))
    o = SparseStorageOptions.from_spec({"sparse_storage_memory_limit_bytes": 1 << 20,
                                        "sparse_storage_spill_dir": str(tmp_path),
                                        "sparse_storage_entries_per_page": 8192})
    assert o.rows_per_page == 8192 and o.memory_limit_bytes == 1 << 20


def test_paged_store_spills_and_round_trips(tmp_path):
    opts = SparseStorageOptions(memory_limit_bytes=4 * 4096 * 4 * 2, spill_directory=str(tmp_path), entries_per_page=4096)
    (st,) = opts.build_stores([("t", 40000, 4, 2, 0.5)], seed=3)  # 10 pages of 4096 rows, 2 resident
    ids = torch.arange(0, 40000, 97)
    first = st.gather(ids)
    assert first[:, :2].abs().max() <= 0.5 and first[:, 2:].abs().max() == 0  # init columns / zero state
    upd = first + torch.arange(ids.numel()).unsqueeze(1).float()
    st.scatter(ids, upd)
    s = st.stats()
    assert s["evictions"] > 0 and s["spill_slots"] > 0 and s["resident_pages"] <= 2
    assert torch.equal(st.gather(ids), upd)  # values survive the spill round trip
    untouched = torch.tensor([1, 4097, 39999])
    assert torch.equal(st.gather(untouched), st.gather(untouched))  # re-initialised pages are deterministic
    assert any(p.name.startswith("worker-") for p in tmp_path.iterdir())


def test_spill_limit_is_enforced(tmp_path):
    opts = SparseStorageOptions(memory_limit_bytes=4096 * 4 * 4, spill_directory=str(tmp_path),
                                max_spill_bytes=4096 * 4 * 4, entries_per_page=4096)
    (st,) = opts.build_stores([("t", 5 * 4096, 4, 4, 0.1)])
    st.scatter(torch.tensor([0]), torch.ones(1, 4))          # page 0 dirty
    st.scatter(torch.tensor([4096]), torch.ones(1, 4))       # evicts page 0 into the only spill slot
    with pytest.raises(RuntimeError, match="max_spill_bytes"):
        st.scatter(torch.tensor([8192]), torch.ones(1, 4))   # page 1 would need a second slot


@pytest.mark.parametrize("kind", ["rowwise_adagrad", "adam"])
def test_paged_collection_equals_the_in_memory_one(tmp_path, kind):
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05)
    tables = [SparseTableSpec("a", 30000, 8, optimizer=opt), SparseTableSpec("b", 9000, 16, pooling="mean", optimizer=opt)]
    B = 64
    opts = SparseStorageOptions(memory_limit_bytes=200_000, spill_directory=str(tmp_path), entries_per_page=4096)
    paged = CpuEmbeddingBagCollection(tables, B, optimizer=opt, storage=opts, seed=1)
    plain = CpuEmbeddingBagCollection(tables, B, optimizer=opt,
                                      weights=[paged.table_weights(f) for f in range(len(tables))])
    g = torch.Generator().manual_seed(0)
    for step in range(4):
        lens = torch.randint(0, 6, (2 * B,), generator=g)
        offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).int()
        vals = torch.cat([torch.randint(0, 30000, (int(lens[:B].sum()),), generator=g),
                          torch.randint(0, 9000, (int(lens[B:].sum()),), generator=g)]).int()
        outs = []
        for c in (paged, plain):
            c.set_input(offs, vals)
            y = c.forward()
            c.backward(torch.ones_like(y) * 0.1 + y * 0.5)
            outs.append(y)
        torch.testing.assert_close(outs[0], outs[1], rtol=0, atol=0)
    for f in range(2):
        torch.testing.assert_close(paged.table_weights(f), plain.table_weights(f), rtol=0, atol=0)
    assert sum(s["evictions"] for s in paged.storage_stats()) > 0
