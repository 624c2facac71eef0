"""CPU sparse ops, planner, collection oracles, native CPU steps and input validation (CPU)."""
import pytest
import torch

from flare_b200.data.synthetic import SCRAMBLE, DLRMSyntheticData, log_uniform_vocab_sizes, make_jagged, zipf_ids
from flare_b200.ops.sparse import CpuSparseEmbeddingOperator, unique_first_occurrence, unique_first_occurrence_reference
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.planner import plan_sharding
from flare_b200.sparse.precision import prepare_sparse_native_gradient, require_finite_sparse_values
from flare_b200.sparse.reference import CpuEmbeddingBagCollection, pool_reference


def test_vocab_sizes_and_zipf():
    v = log_uniform_vocab_sizes()
    assert len(v) == 26 and v[0] == 1000 and v[-1] == 40_000_000 and abs(sum(v) - 2e8) / 2e8 < 0.01
    g = torch.Generator().manual_seed(0)
    ids = zipf_ids(100000, 1000, 1.05, g)
    assert int(ids.min()) >= 0 and int(ids.max()) < 1000
    # the most frequent id is the scrambled rank-0 id and is much hotter than the median
    counts = torch.bincount(ids.long(), minlength=1000)
    assert int(counts.argmax()) == 0 and counts.max() > 20 * counts.median()
    assert SCRAMBLE % 1000 != 0


def test_dlrm_generator_shapes():
    d = DLRMSyntheticData(64, [100, 200, 300], max_bag=5)
    b = d.next()
    assert b.dense.shape == (64, 13) and b.labels.shape == (64, 1)
    assert b.offsets.numel() == 3 * 64 + 1 and int(b.offsets[-1]) == b.values.numel()
    lens = b.offsets[1:] - b.offsets[:-1]
    assert int(lens.min()) >= 1 and int(lens.max()) <= 5


def test_planner_balance_and_rowwise_exactness():
    opt = SparseOptimizerConfig(kind="adam")
    tabs = [SparseTableSpec(f"t{i}", 100 * (i + 1), 128, optimizer=opt) for i in range(26)]
    p = plan_sharding(tabs, 8)
    loads = p.load([1.0] * 26)
    assert max(loads) == min(loads)
    cols = {}
    for pl in p.placements:
        cols.setdefault(pl.table, []).append((pl.col_begin, pl.ncols))
    for t, pieces in cols.items():
        assert sum(n for _, n in pieces) == 128
    rw = [SparseTableSpec(f"t{i}", 100, 128) for i in range(26)]  # row-wise adagrad default
    assert all(pl.ncols == 128 for pl in plan_sharding(rw, 8).placements)
    with pytest.raises(MemoryError):
        plan_sharding([SparseTableSpec("big", 10**9, 128)], 2, hbm_budget_bytes=1e9)


def test_planner_row_wise_pieces():
    """shards=R cuts a table into R modulo pieces spread over ranks; pieces are never column-split."""
    opt = SparseOptimizerConfig(kind="adam")
    tabs = [SparseTableSpec("huge", 10**6 + 3, 128, optimizer=opt, shards=8)] + \
        [SparseTableSpec(f"t{i}", 1000, 64, optimizer=opt) for i in range(4)]
    p = plan_sharding(tabs, 4, expected_lookups=[8.0, 1, 1, 1, 1])
    pieces = [pl for pl in p.placements if pl.table == 0]
    assert sorted(pl.row_index for pl in pieces) == list(range(8))
    assert all(pl.row_shards == 8 and pl.ncols == 128 for pl in pieces)
    assert sorted(pl.rank for pl in pieces) == [0, 0, 1, 1, 2, 2, 3, 3]
    assert sum(pl.num_rows(10**6 + 3) for pl in pieces) == 10**6 + 3
    assert p.row_shards(0) == 8 and p.row_shards(1) == 1
    with pytest.raises(ValueError):
        SparseTableSpec("x", 10, 8, shards=2, cache_rows=5)


def test_reference_pool_matches_bruteforce():
    tabs = [SparseTableSpec("a", 50, 8), SparseTableSpec("b", 30, 8, pooling="mean")]
    g = torch.Generator().manual_seed(1)
    lengths = torch.randint(0, 6, (2, 10), generator=g)
    offs, vals = make_jagged(lengths, [50, 30], 1.1, g)
    ws = [torch.randn(50, 8), torch.randn(30, 8)]
    out = pool_reference(ws, tabs, offs, vals, 10)
    for f in range(2):
        for b in range(10):
            s, e = int(offs[f * 10 + b]), int(offs[f * 10 + b + 1])
            want = ws[f][vals[s:e].long()].sum(0)
            if tabs[f].pooling == "mean" and e > s:
                want = want / (e - s)
            assert torch.allclose(out[b, 8 * f:8 * f + 8], want, atol=1e-6)


def test_reference_rowwise_adagrad_update():
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.1)
    tabs = [SparseTableSpec("a", 10, 4, optimizer=opt)]
    coll = CpuEmbeddingBagCollection(tabs, 2, optimizer=opt, weights=[torch.zeros(10, 4)])
    offs = torch.tensor([0, 2, 3], dtype=torch.int32)
    vals = torch.tensor([3, 3, 5], dtype=torch.int32)
    coll.set_input(offs, vals)
    coll.forward()
    g = torch.tensor([[1.0, 2.0, 3.0, 4.0], [1.0, 1.0, 1.0, 1.0]])
    coll.backward(g, 1)
    # row 3 appears twice in bag 0 -> gradient 2*g0; state = mean(g^2)
    g3 = 2 * g[0]
    s3 = (g3 ** 2).mean()
    assert torch.allclose(coll.weights[0][3], -0.1 * g3 / (s3.sqrt() + 1e-8), atol=1e-6)
    assert torch.allclose(coll.weights[0][5], -0.1 * g[1] / 1.0, atol=1e-6)


def test_padded_cpu_ops_and_unique():
    op = CpuSparseEmbeddingOperator("float32")
    emb = torch.arange(12.0).reshape(4, 3)
    inv = torch.tensor([0, 4, 2, 1], dtype=torch.int32)
    out = op.gather(emb, inv, 2, 3, 4)
    assert torch.equal(out[0, 1], torch.zeros(3)) and torch.equal(out[1, 0], emb[2])
    pooled = op.gather_pooled(emb, inv, 2, 3, (1, 2), 4)
    assert torch.equal(pooled[0, 0], emb[0]) and torch.equal(pooled[1, 0], emb[2] + emb[1])
    sc = op.scatter_pooled(4, 3, inv, 4, torch.ones(2, 1, 3), (1, 2))
    assert torch.equal(sc.sum(1), torch.tensor([3.0, 3.0, 3.0, 0.0]))
    keys = torch.tensor([5, 3, 5, -1, 3, 9])
    u, i, f = unique_first_occurrence(keys)
    ru, ri, rf = unique_first_occurrence_reference(keys)
    assert torch.equal(u, ru) and torch.equal(i, ri) and torch.equal(f, rf)
    assert u.tolist() == [5, 3, -1, 9]


def test_sparse_precision_rescue():
    g = torch.randn(4, 8).to(torch.bfloat16)
    out = prepare_sparse_native_gradient(g, transport_dtype="bfloat16", native_dtype="float32")
    assert out.dtype == torch.float32
    with pytest.raises(TypeError):
        prepare_sparse_native_gradient(g.float(), transport_dtype="bfloat16", native_dtype="float32")
    with pytest.raises(FloatingPointError):
        require_finite_sparse_values(torch.tensor([float("nan")]), "float32", boundary="t")


@pytest.mark.parametrize("dtype,vd", [(torch.float32, "float32"), (torch.float16, "float16")])
def test_native_cpu_ops_match_torch_reference(dtype, vd):
    from flare_b200.ops.sparse import _cpu_native

    if _cpu_native() is None:
        pytest.skip("native extension not built")
    g = torch.Generator().manual_seed(3)
    nat = CpuSparseEmbeddingOperator(vd, use_native=True)
    ref = CpuSparseEmbeddingOperator(vd, use_native=False)
    rows, dim, B, F, E = 300, 32, 16, 4, 6
    emb = torch.randn(rows * dim, generator=g).to(dtype)
    inv = torch.randint(-1, rows, (B * F * E,), generator=g, dtype=torch.int32)
    torch.testing.assert_close(nat.gather(emb, inv, B, dim, -1), ref.gather(emb, inv, B, dim, -1))
    torch.testing.assert_close(nat.gather_pooled(emb, inv, B, dim, (F, E), -1).float(),
                               ref.gather_pooled(emb, inv, B, dim, (F, E), -1).float(), rtol=1e-3, atol=1e-3)
    gp = torch.randn(B * F * dim, generator=g).to(dtype)
    torch.testing.assert_close(nat.scatter_pooled(rows, dim, inv, -1, gp, (F, E)),
                               ref.scatter_pooled(rows, dim, inv, -1, gp, (F, E)), rtol=1e-5, atol=1e-5)
    gs = torch.randn(inv.numel() * dim, generator=g).to(dtype)
    torch.testing.assert_close(nat.scatter(rows, dim, inv, -1, gs), ref.scatter(rows, dim, inv, -1, gs),
                               rtol=1e-5, atol=1e-5)
    keys = torch.randint(0, 97, (2000,), generator=g)
    for a, b in zip(unique_first_occurrence(keys), unique_first_occurrence_reference(keys)):
        assert torch.equal(a, b)


def test_validate_keyed_jagged_catches_bad_batches():
    import pytest
    import torch

    from flare_b200.sparse.collection import validate_keyed_jagged
    from flare_b200.sparse.config import SparseTableSpec

    tables = [SparseTableSpec("a", 10, 8), SparseTableSpec("b", 5, 8, dynamic=True)]
    B = 3
    off = torch.tensor([0, 1, 3, 3, 4, 6, 7], dtype=torch.int32)
    ids = torch.tensor([1, 2, 9, 100, 0, 4, 7], dtype=torch.int32)
    validate_keyed_jagged(off, ids, tables, B, max_bag=4)  # dynamic table b takes any id >= 0
    with pytest.raises(ValueError, match="feature 0"):
        validate_keyed_jagged(off, torch.tensor([1, 2, 10, 100, 0, 4, 7], dtype=torch.int32), tables, B, 4)
    with pytest.raises(ValueError, match="decrease at feature 0, sample 2"):
        validate_keyed_jagged(torch.tensor([0, 1, 3, 2, 4, 6, 7], dtype=torch.int32), ids, tables, B, 4)
    with pytest.raises(ValueError, match="max_bag"):
        validate_keyed_jagged(off, ids, tables, B, max_bag=1)
    with pytest.raises(ValueError, match="end at"):
        validate_keyed_jagged(off, ids[:6], tables, B, 4)
    with pytest.raises(ValueError, match="int32"):
        validate_keyed_jagged(off.long(), ids, tables, B, 4)


def test_native_collection_ops_match_the_tensor_oracle():
    import torch

    from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
    from flare_b200.sparse.reference import CpuEmbeddingBagCollection

    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    tables = [SparseTableSpec("a", 500, 8, optimizer=opt), SparseTableSpec("b", 80, 16, pooling="mean", optimizer=opt),
              SparseTableSpec("c", 300, 4, value_dtype="float16", optimizer=opt)]
    B = 48
    plain = CpuEmbeddingBagCollection(tables, B, optimizer=opt, seed=3)
    fast = CpuEmbeddingBagCollection(tables, B, optimizer=opt, weights=[w.clone() for w in plain.weights],
                                     native=True)
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        lens = torch.randint(0, 7, (3 * B,), generator=g)
        offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).int()
        vals = torch.cat([torch.randint(-1, n, (int(lens[f * B:(f + 1) * B].sum()),), generator=g)
                          for f, n in enumerate((500, 80, 300))]).int()  # -1: skipped ids
        ys = []
        for c in (plain, fast):
            c.set_input(offs, vals)
            y = c.forward()
            c.backward(torch.sin(y) + 0.1)
            ys.append(y)
        torch.testing.assert_close(ys[1], ys[0], rtol=1e-6, atol=1e-6)
    for a, b in zip(plain.weights, fast.weights):
        torch.testing.assert_close(b.float(), a.float(), rtol=1e-5, atol=1e-6)


def test_native_row_optimizer_matches_reference_for_every_kind_and_policy():
    import itertools

    import torch

    from flare_b200._native import native
    from flare_b200.sparse.config import LR_POLICIES, OPTIMIZER_KINDS, SparseOptimizerConfig
    from flare_b200.sparse.reference import apply_rows_reference

    g0 = torch.Generator().manual_seed(0)
    for kind, policy in itertools.product(OPTIMIZER_KINDS, LR_POLICIES):
        opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05, weight_decay=0.01, dynamic_lr_policy=policy,
                                    cosine_max_score=6.0, cosine_min_lr_ratio=0.2,
                                    custom_lut=(1.0, 0.5, 0.25) if policy == "custom_lut" else ())
        R, d = 20, 8
        w0 = torch.randn(R, d, generator=g0)
        st0 = {}
        if opt.needs_row_state:
            st0["row"] = torch.rand(R, generator=g0)
        if opt.needs_m:
            st0["m"] = torch.rand(R, d, generator=g0)
        if opt.needs_v:
            st0["v"] = torch.rand(R, d, generator=g0)
        if opt.needs_score:
            st0["score"] = torch.rand(R, generator=g0) * 3
        rows = torch.tensor([0, 3, 7, 19])
        g = torch.randn(4, d, generator=g0)
        cnt = torch.tensor([1.0, 3.0, 2.0, 5.0])
        for step in (1, 4):
            wa, sa = w0.clone(), {k: v.clone() for k, v in st0.items()}
            wb, sb = w0.clone(), {k: v.clone() for k, v in st0.items()}
            apply_rows_reference(opt, step, wa, rows, g, cnt, sa)
            e = torch.empty(0)
            native().cpu.apply_rows(OPTIMIZER_KINDS[kind], LR_POLICIES[policy],
                                    [opt.learning_rate, opt.beta1, opt.beta2, opt.eps, opt.weight_decay,
                                     opt.cosine_min_lr_ratio, opt.cosine_max_score], list(opt.custom_lut), step,
                                    wb, rows, g, cnt, sb.get("row", e), sb.get("m", e), sb.get("v", e),
                                    sb.get("score", e))
            torch.testing.assert_close(wb, wa, rtol=1e-5, atol=1e-6, msg=f"{kind}/{policy}/step {step}")
            for k in sa:
                torch.testing.assert_close(sb[k], sa[k], rtol=1e-5, atol=1e-6, msg=f"{kind}/{policy} {k}")


def test_staleness_bound_validation():
    import pytest

    from flare_b200.sparse.config import SparseTableSpec

    with pytest.raises(ValueError, match="max_staleness_steps"):
        SparseTableSpec("a", 10, 8, max_staleness_steps=-1)
    assert SparseTableSpec("a", 10, 8, max_staleness_steps=2).max_staleness_steps == 2


def test_exchange_bytes_account_for_the_pipelined_gradient_buffer():
    from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
    from flare_b200.sparse.config import SparseTableSpec

    tabs = [SparseTableSpec("a", 100, 16), SparseTableSpec("b", 50, 8)]
    sync = ShardedEmbeddingBagCollection.exchange_bytes(tabs, 32, 4)
    piped = ShardedEmbeddingBagCollection.exchange_bytes(tabs, 32, 4, pipelined=True)
    assert piped - sync == 4 * 32 * (16 + 8)  # one more [B, total_dim] pooled-gradient buffer


def test_dirty_row_bitmap_unpacking_without_cuda():
    """Dirty rows live in a bitmap of 32 rows per int32 word (bit 31 included); ranges may start and
    end inside a word."""
    import torch

    from flare_b200.sparse.collection import ShardedEmbeddingBagCollection

    c = object.__new__(ShardedEmbeddingBagCollection)
    c.device = torch.device("cpu")
    c.num_local_rows = 100
    c.dirty_bits = torch.zeros(4, dtype=torch.int32)
    rows = [0, 5, 31, 32, 63, 64, 70, 99]
    for r in rows:
        w = int(c.dirty_bits[r // 32]) & 0xFFFFFFFF
        w |= 1 << (r % 32)
        c.dirty_bits[r // 32] = w - (1 << 32) if w >= 1 << 31 else w
    assert c.dirty_rows(0, 100).tolist() == rows
    assert c.dirty_rows(30, 40).tolist() == [1, 2, 33, 34]  # rows 31, 32, 63, 64 relative to 30
    assert c.dirty.nonzero().flatten().tolist() == rows
    c.clear_dirty()
    assert c.dirty_rows(0, 100).numel() == 0
