"""Gradient-accumulation windows on the fused path (one GPU).

A window of n micro-batches must equal one optimizer step on their union
with the gradient divided by n: checked on the sharded collection against a
collection of n times the batch, and on the fused DLRM against the plain
PyTorch model accumulating gradients over the same micro-batches.
"""
import pytest
import torch

from flare_b200.data.synthetic import DLRMSyntheticData, make_jagged
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["hash", "sorted", "hash_staged"])
def bwd_path(request, monkeypatch):
    if request.param == "sorted":
        monkeypatch.setenv("FLARE_EMB_LEGACY_BWD", "1")
    if request.param == "hash_staged":
        monkeypatch.setenv("FLARE_EMB_GRAD_STAGE", "1")
    return request.param


def _batch(B, vocabs, max_bag, seed):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(0, max_bag + 1, (len(vocabs), B), generator=g)
    return make_jagged(lengths, vocabs, 1.05, g)


def _union(batches, F, B):
    """Keyed-jagged batch of the micro-batches' samples, micro-batch k's samples at k*B.. of every feature."""
    offs, vals, base = [0], [], 0
    for f in range(F):
        for o, v in batches:
            seg = o[f * B:(f + 1) * B + 1].long()
            vals.append(v[seg[0]:seg[-1]])
            offs.extend((seg[1:] - seg[0] + base).tolist())
            base += int(seg[-1] - seg[0])
    return torch.tensor(offs, dtype=torch.int32), torch.cat(vals)


@pytest.mark.parametrize("kind", ["rowwise_adagrad", "adam", "sgd"])
@pytest.mark.parametrize("micro", [3, 2])
def test_window_equals_one_step_on_the_union(cuda, kind, micro, bwd_path):
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05, weight_decay=0.001)
    vocabs = [500, 3000, 40]
    tables = [SparseTableSpec("a", vocabs[0], 32, optimizer=opt),
              SparseTableSpec("b", vocabs[1], 64, optimizer=opt, pooling="mean"),
              SparseTableSpec("c", vocabs[2], 16, optimizer=opt)]
    B, max_bag, n = 128, 6, 3
    kw = dict(max_bag_size=max_bag, device=cuda, optimizer=opt, seed=3, grad_dtype=torch.float32, light_max=3)
    win = ShardedEmbeddingBagCollection(tables, B, accumulation_steps=n, **kw)
    ref = ShardedEmbeddingBagCollection(tables, n * B, **kw)
    torch.testing.assert_close(win.weights, ref.weights, rtol=0, atol=0)
    assert win.hash_bwd == (bwd_path != "sorted")
    for window in range(2):
        batches = [_batch(B, vocabs, max_bag, seed=10 * window + k) for k in range(micro)]
        grads = [torch.randn(B, win.total_dim, device=cuda) * 0.1 for _ in range(micro)]
        for (o, v), g in zip(batches, grads):
            win.set_input(o.to(cuda), v.to(cuda), non_blocking=False)
            pooled = win.forward()
            win.grad_input.copy_(g)
        assert win.micro_filled == micro
        win.backward()  # micro < n: a tail window, normalised by its own count
        assert win.micro_filled == 0
        # the union, padded with empty samples up to n * B, one step with the window-mean gradient
        empty = (torch.zeros(len(vocabs) * B + 1, dtype=torch.int32), torch.zeros(0, dtype=torch.int32))
        o, v = _union(batches + [empty] * (n - micro), len(vocabs), B)
        ref.set_input(o.to(cuda), v.to(cuda), non_blocking=False)
        pooled_ref = ref.forward()
        torch.testing.assert_close(pooled_ref[(micro - 1) * B:micro * B].float(), pooled.float(), rtol=1e-2, atol=1e-3)
        g = torch.cat(grads + [torch.zeros_like(grads[0])] * (n - micro)) / micro
        ref.grad_input.copy_(g)
        ref.backward()
        torch.cuda.synchronize()
        win.check()
        ref.check()
        # the window and the union add a row's gradients in another fp32 order; Adam divides by the
        # gradient's own magnitude, so a row whose gradients nearly cancel can move by up to the
        # learning rate on that rounding: allow 0.1 % of elements outside the tolerance
        def close(a, b, rtol, atol):
            bad = (a - b).abs() > atol + rtol * b.abs()
            assert float(bad.float().mean()) < 1e-3 and float((a - b).abs().max()) <= 2 * opt.learning_rate, \
                (int(bad.sum()), float((a - b).abs().max()))

        close(win.weights, ref.weights, 1e-5, 1e-6)
        for name in ("state_row", "state_m", "state_v"):
            a, b = getattr(win, name), getattr(ref, name)
            if a is not None:
                close(a, b, 1e-4, 1e-7)
    assert win.step == ref.step == 2


def test_window_guards(cuda):
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    tables = [SparseTableSpec("a", 100, 32, optimizer=opt)]
    c = ShardedEmbeddingBagCollection(tables, 16, max_bag_size=4, device=cuda, accumulation_steps=2)
    with pytest.raises(RuntimeError, match="no micro-step"):
        c.backward()
    o, v = _batch(16, [100], 4, 1)
    c.set_input(o.to(cuda), v.to(cuda), non_blocking=False)
    c.forward()
    c.forward()
    with pytest.raises(RuntimeError, match="holds 2 micro-steps"):
        c.forward()
    c.forward(training=False)  # evaluation lookups stage nothing
    with pytest.raises(ValueError, match="accumulation windows"):
        ShardedEmbeddingBagCollection(tables, 16, max_bag_size=4, device=cuda, accumulation_steps=2, pipelined=True)


VOCABS = [200, 3000, 50, 10000, 700]


def test_dlrm_window_tracks_pytorch_accumulation(cuda):
    """Fused DLRM with 3-micro-step windows (graph replay, one graph per position) against the plain
    PyTorch model that backpropagates loss / 3 of each micro-batch and steps at the window end."""
    from flare_b200.models.dlrm import DLRMConfig, DLRMTorch, RowwiseAdagradTorch, dlrm_benchmark_tables
    from flare_b200.training.trainer import DLRMTrainer

    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    cfg = DLRMConfig(tables=dlrm_benchmark_tables(VOCABS, 64, opt), bottom=(128, 64), top=(256, 128),
                     sparse_optimizer=opt)
    B, n = 256, 3
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, device=cuda, seed=31, pos_rate=0.3)
    batches = [data.next() for _ in range(8 * n + 2)]
    tr = DLRMTrainer(cfg, B, max_bag_size=8, device=cuda, seed=9, use_graph=True, accumulation_steps=n)
    ref = DLRMTorch(cfg).to(cuda).load_from_fused(tr.model)
    dense = [p for name, p in ref.named_parameters() if not name.startswith("embs.")]
    opt_d = torch.optim.Adam(dense, lr=cfg.dense_optimizer.learning_rate, betas=(0.9, 0.999), eps=1e-8)
    opt_s = RowwiseAdagradTorch([e.weight for e in ref.embs], lr=0.05, eps=cfg.sparse_optimizer.eps)
    fused, plain = [], []
    for i, b in enumerate(batches):
        fused.append(tr.train_step(b).loss)
        logits = ref(b.dense, b.offsets, b.values)
        loss = torch.nn.functional.binary_cross_entropy_with_logits(logits.view(-1), b.labels.view(-1).float())
        (loss / (n if i < 8 * n else 2)).backward()
        plain.append(float(loss.detach()))
        if (i + 1) % n == 0 and i < 8 * n:
            opt_d.step()
            opt_s.step()
            opt_d.zero_grad(set_to_none=True)
            opt_s.zero_grad()
    assert len(tr.graphs) == n and tr.model.emb.step == 8 and tr.model.emb.micro_filled == 2
    assert tr.flush_pending_updates() and not tr.flush_pending_updates()  # the 2-micro-step tail window
    opt_d.step()
    opt_s.step()
    assert tr.model.emb.step == 9 and tr.model.dense.step == 9
    tr.check()
    for i, (a, p) in enumerate(zip(fused, plain)):
        assert abs(a - p) <= 0.03 * abs(p) + 2e-3, (i, fused, plain)
    # after the tail window: the loss of held-out batches under both models (the tail update included)
    held = [data.next() for _ in range(3)]
    for b in held:
        tr.model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=False)
        p = tr.model.predict().view(-1).double().clamp(1e-6, 1 - 1e-6)
        y = b.labels.view(-1).double()
        fused_loss = float(-(y * p.log() + (1 - y) * (1 - p).log()).mean())
        with torch.no_grad():
            logits = ref(b.dense, b.offsets, b.values).view(-1)
            plain_loss = float(torch.nn.functional.binary_cross_entropy_with_logits(logits, y.float()))
        assert abs(fused_loss - plain_loss) <= 0.03 * plain_loss + 2e-3, (fused_loss, plain_loss)
