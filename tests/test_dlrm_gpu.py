"""End-to-end fused DLRM on one GPU: forward equivalence, training progress, graph replay."""
import pytest
import torch

from flare_b200.data.synthetic import DLRMSyntheticData
from flare_b200.models.dlrm import DLRM, DLRMConfig, DLRMTorch, dlrm_benchmark_tables
from flare_b200.sparse.config import SparseOptimizerConfig
from flare_b200.training.trainer import DLRMTrainer

pytestmark = pytest.mark.gpu

VOCABS = [200, 3000, 50, 10000, 700]


def _cfg(lr_sparse=0.05):
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=lr_sparse)
    return DLRMConfig(tables=dlrm_benchmark_tables(VOCABS, 64, opt), bottom=(128, 64), top=(256, 128),
                      sparse_optimizer=opt)


def test_forward_matches_torch(cuda):
    cfg = _cfg()
    B = 256
    model = DLRM(cfg, B, max_bag_size=12, device=cuda, seed=1)
    data = DLRMSyntheticData(B, VOCABS, max_bag=12, device=cuda, seed=2)
    b = data.next()
    model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=False)
    probs = model.predict()
    ref = DLRMTorch(cfg).to(cuda).load_from_fused(model)
    with torch.no_grad():
        ref_logits = ref(b.dense, b.offsets, b.values)
    torch.testing.assert_close(probs, torch.sigmoid(ref_logits), rtol=0.05, atol=0.02)


def test_training_reduces_loss_and_graph_matches_eager(cuda):
    cfg = _cfg()
    B = 512
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, device=cuda, seed=3, pos_rate=0.3)
    batches = [data.next() for _ in range(4)]
    losses = {}
    for use_graph in (False, True):
        tr = DLRMTrainer(cfg, B, max_bag_size=8, device=cuda, seed=5, use_graph=use_graph)
        seq = [tr.train_step(batches[i % 4]).loss for i in range(40)]
        tr.check()
        losses[use_graph] = seq
        if use_graph:
            assert tr.graph is not None and tr.launches_per_step > 10
    eager, graph = losses[False], losses[True]
    assert sum(eager[-8:]) / 8 < sum(eager[:4]) / 4
    # float atomics in the sparse and split-K reductions make two runs differ in the last bits; the
    # difference compounds while training overfits the four batches, so later steps get a looser bound
    # (a replay bug shows at once: the first replayed step is step 2)
    for i, (a, b) in enumerate(zip(eager, graph)):
        tol = 3e-3 * max(1.0, abs(a)) if i < 16 else 3e-2 * abs(a) + 1e-3
        assert abs(a - b) <= tol, (i, a, b)


@pytest.mark.parametrize("staleness", [1, 2])
def test_pipelined_policy_matches_stale_emulation(cuda, staleness):
    """Pipelined steps equal sync steps whose lookups read the tables ``staleness`` sparse updates behind."""
    cfg = _cfg(lr_sparse=0.05)
    B, d = 256, staleness
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, device=cuda, seed=11, pos_rate=0.3)
    batches = [data.next() for _ in range(8)]
    tr = DLRMTrainer(cfg, B, max_bag_size=8, device=cuda, seed=4, use_graph=True, sparse_policy="pipelined",
                     staleness=d)
    piped = [tr.train_step(b).loss for b in batches]
    # d updates in flight; the slots rotate over d + 1 buffers: one graph per position
    assert len(tr.model.pending) == d and len(tr.graphs) == d + 1
    assert tr.flush_pending_updates() and not tr.flush_pending_updates()
    tr.check()

    ref = DLRM(cfg, B, max_bag_size=8, device=cuda, seed=4)
    hist, emulated = [ref.emb.weights.clone()], []  # hist[k]: tables after the updates of steps < k
    for t, b in enumerate(batches):
        ref.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=False)
        cur = ref.emb.weights.clone()
        ref.emb.weights.copy_(hist[max(t - d, 0)])  # lookups miss the updates of steps t-d .. t-1
        loss = ref.forward_backward()
        ref.emb.weights.copy_(cur)
        ref.emb.backward()
        ref.dense.apply()
        emulated.append(float(loss.item()) / B)
        hist.append(ref.emb.weights.clone())
    ref.check()
    for a, b in zip(piped, emulated):
        assert abs(a - b) <= 1e-3 * max(1.0, abs(a)), (piped, emulated)
    torch.testing.assert_close(tr.model.emb.weights, ref.emb.weights, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(tr.model.dense.master, ref.dense.master, rtol=1e-3, atol=1e-4)
    tr.close()


def test_loss_trajectory_tracks_pytorch_model_over_24_steps(cuda):
    """The fused DLRM (graph replay, bf16 compute, fused row-wise Adagrad + Adam) and the plain
    PyTorch model (fp32, nn.EmbeddingBag + RowwiseAdagradTorch + torch.optim.Adam) start from the
    same weights and train on 24 distinct batches: their per-step losses stay together."""
    from flare_b200.models.dlrm import RowwiseAdagradTorch

    cfg = _cfg(lr_sparse=0.05)
    B = 512
    data = DLRMSyntheticData(B, VOCABS, max_bag=8, device=cuda, seed=21, pos_rate=0.3)
    batches = [data.next() for _ in range(24)]
    tr = DLRMTrainer(cfg, B, max_bag_size=8, device=cuda, seed=9, use_graph=True)
    ref = DLRMTorch(cfg).to(cuda).load_from_fused(tr.model)
    dense = [p for n, p in ref.named_parameters() if not n.startswith("embs.")]
    opt_d = torch.optim.Adam(dense, lr=cfg.dense_optimizer.learning_rate, betas=(0.9, 0.999), eps=1e-8)
    opt_s = RowwiseAdagradTorch([e.weight for e in ref.embs], lr=0.05, eps=cfg.sparse_optimizer.eps)
    fused, plain = [], []
    for b in batches:
        fused.append(tr.train_step(b).loss)
        logits = ref(b.dense, b.offsets, b.values)
        loss = torch.nn.functional.binary_cross_entropy_with_logits(logits.view(-1), b.labels.view(-1).float())
        opt_d.zero_grad(set_to_none=True)
        opt_s.zero_grad()
        loss.backward()
        opt_d.step()
        opt_s.step()
        plain.append(float(loss))
    tr.check()
    for i, (a, p) in enumerate(zip(fused, plain)):
        assert abs(a - p) <= 0.03 * abs(p) + 2e-3, (i, fused, plain)
    assert sum(plain[-6:]) < sum(plain[:6])  # both learn (distinct batches, not memorised)
