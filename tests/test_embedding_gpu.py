"""Fused sharded embedding collection (world size 1) vs the CPU reference store."""
import pytest
import torch

from flare_b200.data.synthetic import make_jagged
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.planner import ShardingPlan, ShardPlacement
from flare_b200.sparse.reference import CpuEmbeddingBagCollection

pytestmark = pytest.mark.gpu


def _batch(B, vocabs, max_bag, seed, zipf=1.05):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(0, max_bag + 1, (len(vocabs), B), generator=g)
    return make_jagged(lengths, vocabs, zipf, g)


def _export(coll, tables):
    """Full host tables assembled from the GPU shards."""
    ws = [torch.zeros(t.num_embeddings, t.embedding_dim) for t in tables]
    for i, s in enumerate(coll.shards):
        ws[s.table][s.row_slice, s.col_begin:s.col_begin + s.ncols] = coll.shard_view(i).float().cpu()
    return ws


class _PieceReference:
    """CPU reference where every column shard is an independent table."""

    def __init__(self, tables, coll, opt):
        self.tables, self.pieces = tables, [(s.table, s.col_begin, s.ncols) for s in coll.shards]
        full = _export(coll, tables)
        specs = [SparseTableSpec(f"p{i}", tables[t].num_embeddings, n, optimizer=opt, pooling=tables[t].pooling,
                                 feature=f"p{i}") for i, (t, c, n) in enumerate(self.pieces)]
        self.inner = CpuEmbeddingBagCollection(specs, coll.B, optimizer=opt,
                                               weights=[full[t][:, c:c + n].clone() for t, c, n in self.pieces])
        self.B = coll.B

    def _expand(self, offs, vals):
        B = self.B
        o, v, base = [0], [], 0
        for t, _, _ in self.pieces:
            seg = offs[t * B:(t + 1) * B + 1].long()
            v.append(vals[seg[0]:seg[-1]])
            o.extend((seg[1:] - seg[0] + base).tolist())
            base += int(seg[-1] - seg[0])
        return torch.tensor(o, dtype=torch.int32), torch.cat(v)

    def set_input(self, offs, vals):
        self.inner.set_input(*self._expand(offs, vals))

    def forward(self):
        out = self.inner.forward()
        res = torch.zeros(self.B, sum(t.embedding_dim for t in self.tables))
        col, starts = 0, []
        for t in self.tables:
            starts.append(col)
            col += t.embedding_dim
        k = 0
        for t, c, n in self.pieces:
            res[:, starts[t] + c:starts[t] + c + n] = out[:, k:k + n]
            k += n
        return res

    def backward(self, grad, step):
        starts, col = [], 0
        for t in self.tables:
            starts.append(col)
            col += t.embedding_dim
        g = torch.cat([grad[:, starts[t] + c:starts[t] + c + n] for t, c, n in self.pieces], 1)
        self.inner.backward(g, step)

    @property
    def weights(self):
        ws = [torch.zeros(t.num_embeddings, t.embedding_dim) for t in self.tables]
        for (t, c, n), w in zip(self.pieces, self.inner.weights):
            ws[t][:, c:c + n] = w
        return ws


def _cw_plan(tables):
    pl, out, c = [], [], 0
    for i, t in enumerate(tables):
        out.append(c)
        c += t.embedding_dim
        half = t.embedding_dim // 2
        pl += [ShardPlacement(i, 0, half, 0), ShardPlacement(i, half, half, 0)]
    return ShardingPlan(1, tuple(pl), tuple(out), c)


def _assert_scratch_clean(coll):
    """Every backward leaves its dedup scratch as it found it (hash table empty / row counters zero)."""
    if coll.hash_bwd:
        assert bool((coll.htab == 0xFFFFFFFF).all())
    else:
        assert int(coll.row_count.abs().max()) == 0


@pytest.fixture(params=["hash", "sorted", "hash_staged"])
def bwd_path(request, monkeypatch):
    """The hash-dedup backward (gradients read in place, or pulled into the staging buffer as on several
    GPUs) and the sorted per-row backward."""
    if request.param == "sorted":
        monkeypatch.setenv("FLARE_EMB_LEGACY_BWD", "1")
    if request.param == "hash_staged":
        monkeypatch.setenv("FLARE_EMB_GRAD_STAGE", "1")
    return request.param


@pytest.mark.parametrize("kind", ["rowwise_adagrad", "adam", "sgd", "adagrad", "rowwise_adam"])
@pytest.mark.parametrize("split", ["none", "column", "row"])
def test_forward_backward_matches_reference(cuda, kind, split, bwd_path):
    torch.manual_seed(0)
    column_split = split == "column"
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05, weight_decay=0.001)
    vocabs = [50, 1000, 7]
    # row: tables 0 and 1 cut into 3 modulo pieces (all owned by this rank), fp32 partials summed
    tables = [SparseTableSpec(f"t{i}", v, 64, optimizer=opt, pooling="mean" if i == 1 else "sum",
                              shards=3 if split == "row" and i < 2 else 1)
              for i, v in enumerate(vocabs)]
    B, max_bag = 96, 20
    plan = _cw_plan(tables) if column_split else None
    coll = ShardedEmbeddingBagCollection(tables, B, max_bag_size=max_bag, device=cuda, plan=plan, optimizer=opt,
                                         seed=3, light_max=3)
    assert coll.hash_bwd == (bwd_path != "sorted")
    assert coll.grad_direct == (bwd_path == "hash")
    ref = CpuEmbeddingBagCollection(tables, B, optimizer=opt, weights=_export(coll, tables))
    split_ref = column_split and opt.needs_row_state
    if split_ref:
        # Row-wise optimizer state is kept per (row, column shard): model every
        # column piece as its own table in the reference.
        ref = _PieceReference(tables, coll, opt)
    for step in range(1, 4):
        offs, vals = _batch(B, vocabs, max_bag, seed=step)
        coll.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
        ref.set_input(offs, vals)
        pooled = coll.forward()
        pooled_ref = ref.forward()
        torch.testing.assert_close(pooled.float().cpu(), pooled_ref.to(torch.bfloat16).float(), rtol=2e-2, atol=1e-3)
        grad = (torch.randn(B, coll.total_dim) * 0.1).to(torch.bfloat16)
        coll.grad_input.copy_(grad.to(cuda))
        coll.backward(step)
        ref.backward(grad.float(), step)
        torch.cuda.synchronize()
        coll.check()
        for w_gpu, w_ref in zip(_export(coll, tables), ref.weights):
            torch.testing.assert_close(w_gpu, w_ref, rtol=1e-4, atol=1e-5)
    _assert_scratch_clean(coll)


def test_hot_rows_heavy_path(cuda, bwd_path):
    """A few rows hit thousands of times (Zipf head): chunked across warps, partials added in order."""
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.1)
    tables = [SparseTableSpec("hot", 4, 128, optimizer=opt)]
    B, max_bag = 512, 32
    coll = ShardedEmbeddingBagCollection(tables, B, max_bag_size=max_bag, device=cuda, optimizer=opt)
    ref = CpuEmbeddingBagCollection(tables, B, optimizer=opt, weights=_export(coll, tables))
    offs, vals = _batch(B, [4], max_bag, seed=11)
    coll.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
    ref.set_input(offs, vals)
    coll.forward()
    grad = torch.randn(B, 128).to(torch.bfloat16)
    coll.grad_input.copy_(grad.to(cuda))
    coll.backward(1)
    ref.backward(grad.float(), 1)
    torch.cuda.synchronize()
    coll.check()
    torch.testing.assert_close(_export(coll, tables)[0], ref.weights[0], rtol=1e-4, atol=1e-5)
    assert int(coll.num_unique[2]) > 0  # the heavy path ran
    if coll.hash_bwd:
        assert int(coll.num_unique[3]) > 4  # rows of more than 256 occurrences were cut into several chunks
    _assert_scratch_clean(coll)


def test_lr_policies(cuda):
    for pol, extra in [("sqrt_decay", {}), ("cosine_frequency", dict(cosine_min_lr_ratio=0.1, cosine_max_score=50.0)),
                       ("custom_lut", dict(custom_lut=(1.0, 0.5, 0.25))), ("log_decay", {}), ("inverse_decay", {})]:
        opt = SparseOptimizerConfig(kind="sgd", learning_rate=0.5, dynamic_lr_policy=pol, **extra)
        tables = [SparseTableSpec("t", 30, 32, optimizer=opt)]
        coll = ShardedEmbeddingBagCollection(tables, 16, max_bag_size=8, device=cuda, optimizer=opt)
        ref = CpuEmbeddingBagCollection(tables, 16, optimizer=opt, weights=_export(coll, tables))
        for step in (1, 2):
            offs, vals = _batch(16, [30], 8, seed=20 + step)
            coll.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
            ref.set_input(offs, vals)
            coll.forward()
            grad = torch.randn(16, 32).to(torch.bfloat16)
            coll.grad_input.copy_(grad.to(cuda))
            coll.backward(step)
            ref.backward(grad.float(), step)
        torch.cuda.synchronize()
        torch.testing.assert_close(_export(coll, tables)[0], ref.weights[0], rtol=1e-4, atol=1e-5, msg=pol)


def test_row_wise_pieces_init_and_pooling(cuda):
    """Modulo row pieces reproduce the whole table's init and its pooled rows (partials summed in fp32)."""
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    vocabs = [1001, 37]
    whole = [SparseTableSpec(f"t{i}", v, 128, optimizer=opt) for i, v in enumerate(vocabs)]
    cut = [SparseTableSpec(f"t{i}", v, 128, optimizer=opt, shards=4) for i, v in enumerate(vocabs)]
    B, max_bag = 64, 12
    a = ShardedEmbeddingBagCollection(whole, B, max_bag_size=max_bag, device=cuda, seed=5)
    b = ShardedEmbeddingBagCollection(cut, B, max_bag_size=max_bag, device=cuda, seed=5)
    assert len(b.shards) == 8 and b.rw_slots == 4
    for wa, wb in zip(_export(a, whole), _export(b, cut)):
        assert torch.equal(wa, wb)
    offs, vals = _batch(B, vocabs, max_bag, seed=9)
    for c in (a, b):
        c.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
    pa, pb = a.forward().float(), b.forward().float()
    torch.cuda.synchronize()
    a.check()
    b.check()
    torch.testing.assert_close(pb, pa, rtol=1e-2, atol=1e-4)


def test_deterministic_mode_is_bitwise_repeatable(cuda):
    """FLARE_DETERMINISTIC: heavy-hitter batches give bitwise-identical tables on repeated runs."""
    opt = SparseOptimizerConfig(kind="adam", learning_rate=0.01)
    vocabs = [40, 5000]
    tables = [SparseTableSpec(f"t{i}", v, 128, optimizer=opt) for i, v in enumerate(vocabs)]
    B, max_bag = 512, 32
    runs = []
    for _ in range(2):
        coll = ShardedEmbeddingBagCollection(tables, B, max_bag_size=max_bag, device=cuda, optimizer=opt, seed=1,
                                             deterministic=True)
        for step in range(1, 4):
            offs, vals = _batch(B, vocabs, max_bag, seed=100 + step, zipf=1.3)
            coll.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
            coll.forward()
            g = torch.Generator().manual_seed(step)
            coll.grad_input.copy_((torch.randn(B, coll.total_dim, generator=g) * 0.1).to(torch.bfloat16).to(cuda))
            coll.backward(step)
        torch.cuda.synchronize()
        coll.check()
        assert coll.last_step_stats()["heavy_rows"] > 0
        runs.append(_export(coll, tables))
    for a, b in zip(*runs):
        assert torch.equal(a, b)


def test_many_unique_rows_across_tiles(cuda, bwd_path):
    """Tens of thousands of distinct rows: many counting tiles, many scan tiles chained by look-back,
    light, single-chunk and multi-chunk rows in one step; two steps so the emptied table is reused."""
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    vocabs = [200_000, 3_000]
    tables = [SparseTableSpec(f"t{i}", v, 128, optimizer=opt) for i, v in enumerate(vocabs)]
    B, max_bag = 2048, 32
    coll = ShardedEmbeddingBagCollection(tables, B, max_bag_size=max_bag, device=cuda, optimizer=opt, seed=2)
    ref = CpuEmbeddingBagCollection(tables, B, optimizer=opt, weights=_export(coll, tables))
    for step in (1, 2):
        offs, vals = _batch(B, vocabs, max_bag, seed=40 + step, zipf=1.05)
        coll.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
        ref.set_input(offs, vals)
        coll.forward()
        ref.forward()
        grad = (torch.randn(B, coll.total_dim) * 0.1).to(torch.bfloat16)
        coll.grad_input.copy_(grad.to(cuda))
        coll.backward(step)
        ref.backward(grad.float(), step)
        torch.cuda.synchronize()
        coll.check()
        stats = coll.last_step_stats()
        assert stats["unique_rows"] > 5000 and stats["heavy_rows"] > 0
        for w_gpu, w_ref in zip(_export(coll, tables), ref.weights):
            torch.testing.assert_close(w_gpu, w_ref, rtol=1e-4, atol=1e-5)
    _assert_scratch_clean(coll)
