"""Checkpoint / resume of the fused DLRM: exact resume, incremental chains, resharding, inference assets."""
from dataclasses import replace

import pytest
import torch

from flare_b200.checkpoint.inference import bind_inference_weights
from flare_b200.checkpoint.store import CheckpointManager, list_steps
from flare_b200.data.synthetic import DLRMSyntheticData
from flare_b200.models.dlrm import DLRM, DLRMConfig, dlrm_benchmark_tables
from flare_b200.sparse.config import SparseOptimizerConfig
from flare_b200.sparse.planner import ShardingPlan, ShardPlacement

pytestmark = pytest.mark.gpu
VOCABS = [300, 5000, 64]


def _cfg(kind="adam", row_shards=(1, 1, 1)):
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05)
    tables = [replace(t, shards=r) for t, r in zip(dlrm_benchmark_tables(VOCABS, 64, opt), row_shards)]
    return DLRMConfig(tables=tables, bottom=(128, 64), top=(128, 64), sparse_optimizer=opt)


def _step(model, batch):
    model.set_batch(batch.dense, batch.labels, batch.offsets, batch.values, non_blocking=False)
    return float(model.train_step().item())


def _tables(model):
    return dict(enumerate(model.emb.assemble_tables(model.emb.export_pieces(), model.emb.tables)))


def test_resume_is_exact_and_incremental_chain(cuda, tmp_path):
    data = DLRMSyntheticData(128, VOCABS, max_bag=8, device=cuda, seed=1)
    batches = [data.next() for _ in range(6)]
    a = DLRM(_cfg(), 128, max_bag_size=8, device=cuda, seed=3)
    mgr = CheckpointManager(str(tmp_path))
    for b in batches[:2]:
        _step(a, b)
    mgr.save(2, a)
    _step(a, batches[2])
    mgr.save(3, a, incremental=True)   # only rows touched by step 3
    losses_a = [_step(a, b) for b in batches[3:]]
    assert list_steps(tmp_path) == [2, 3]
    # resume from the incremental step into a model whose column split differs (reshard on load)
    pl, outc, c = [], [], 0
    for i in range(len(VOCABS)):
        outc.append(c)
        c += 64
        pl += [ShardPlacement(i, 0, 32, 0), ShardPlacement(i, 32, 32, 0)]
    b_model = DLRM(_cfg(), 128, max_bag_size=8, device=cuda, seed=99)
    b_model.emb.__init__(b_model.cfg.tables, 128, max_bag_size=8, device=cuda, optimizer=b_model.cfg.sparse_optimizer,
                         plan=ShardingPlan(1, tuple(pl), tuple(outc), c))
    assert mgr.restore(b_model) == 3
    losses_b = [_step(b_model, b) for b in batches[3:]]
    torch.cuda.synchronize()
    for x, y in zip(losses_a, losses_b):
        assert abs(x - y) <= 1e-3 * max(1.0, abs(x))
    ta, tb = _tables(a), _tables(b_model)
    for t in ta:
        torch.testing.assert_close(ta[t], tb[t], rtol=1e-4, atol=1e-5)


def test_inference_asset_binding(cuda, tmp_path):
    a = DLRM(_cfg("rowwise_adagrad"), 64, max_bag_size=4, device=cuda, seed=5)
    CheckpointManager(str(tmp_path)).save(1, a)
    w = bind_inference_weights(tmp_path, 1)
    b = DLRM(_cfg("rowwise_adagrad"), 64, max_bag_size=4, device=cuda, seed=6)
    w.load_model(b.dense)
    w.load_sparse(b.emb)
    torch.testing.assert_close(b.dense.master, a.dense.master)
    ta, tb = _tables(a), _tables(b)
    for t in ta:
        assert torch.equal(ta[t], tb[t])
    (w.path / "model" / "extra.npy").write_bytes(b"x")  # mutate the published asset
    with pytest.raises(RuntimeError):
        w.verify()


@pytest.mark.parametrize("src,dst", [((3, 2, 1), (1, 1, 1)), ((1, 1, 1), (2, 3, 1))])
def test_row_wise_pieces_reshard(cuda, tmp_path, src, dst):
    """Row-wise (modulo) pieces: same init as whole tables, exact resume into another row split."""
    data = DLRMSyntheticData(128, VOCABS, max_bag=8, device=cuda, seed=4)
    batches = [data.next() for _ in range(5)]
    a = DLRM(_cfg("rowwise_adagrad", src), 128, max_bag_size=8, device=cuda, seed=3)
    ref = DLRM(_cfg("rowwise_adagrad"), 128, max_bag_size=8, device=cuda, seed=3)
    ta, tr = _tables(a), _tables(ref)
    for t in ta:
        assert torch.equal(ta[t], tr[t])   # counter-based init reproduces every row in any split
    mgr = CheckpointManager(str(tmp_path))
    _step(a, batches[0])
    mgr.save(1, a)
    _step(a, batches[1])
    mgr.save(2, a, incremental=True)
    losses_a = [_step(a, b) for b in batches[2:]]
    b_model = DLRM(_cfg("rowwise_adagrad", dst), 128, max_bag_size=8, device=cuda, seed=77)
    assert mgr.restore(b_model) == 2
    # the restored state, saved again from the other split, audits to the same digests
    from flare_b200.checkpoint.audit import audit_step

    CheckpointManager(str(tmp_path / "again")).save(2, b_model)
    ra, rb = audit_step(tmp_path, 2), audit_step(tmp_path / "again", 2)
    assert ra["ok"] and rb["ok"] and ra["sparse"]["chain"] == [1, 2]
    assert ra["sparse"]["digest"] == rb["sparse"]["digest"] and ra["dense"]["digest"] == rb["dense"]["digest"]
    losses_b = [_step(b_model, b) for b in batches[2:]]
    torch.cuda.synchronize()
    for x, y in zip(losses_a, losses_b):
        assert abs(x - y) <= 1e-3 * max(1.0, abs(x))
    ta, tb = _tables(a), _tables(b_model)
    for t in ta:
        torch.testing.assert_close(ta[t], tb[t], rtol=1e-4, atol=1e-5)
