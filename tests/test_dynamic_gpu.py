"""Dynamic (hash-keyed) tables: insert on first sight with the documented init, training
matches a host dict-based store (no eviction), and eviction + rebuild keep lookups consistent."""
import numpy as np
import pytest
import torch

from flare_b200.data.synthetic import zipf_ids
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.dynamic import uniform_init_reference

pytestmark = pytest.mark.gpu
KEY_SPACE = 1_000_000_000


def _kjt(B, max_bag, g):
    ln = torch.randint(1, max_bag + 1, (B,), generator=g)
    vals = zipf_ids(int(ln.sum()), KEY_SPACE, 1.05, g)
    off = torch.zeros(B + 1, dtype=torch.int32)
    torch.cumsum(ln, 0, out=off[1:])
    return off, vals


def _ref_row(store, seed, key, dim, scale):
    if key not in store:
        store[key] = np.array([(2 * uniform_init_reference(seed, key, c) - 1) * scale for c in range(dim)],
                              dtype=np.float64)
    return store[key]


def test_dynamic_table_matches_dict_store(cuda):
    dim, scale, lr = 64, 0.01, 0.1
    opt = SparseOptimizerConfig(kind="sgd", learning_rate=lr)
    spec = SparseTableSpec("d", 8192, dim, optimizer=opt, dynamic=True, init_scale=scale)
    B, bag = 128, 6
    coll = ShardedEmbeddingBagCollection([spec], B, max_bag_size=bag, device=cuda, optimizer=opt, seed=5)
    ds = coll.dynamic.shards[0]
    store = {}
    g = torch.Generator().manual_seed(1)
    for step in range(5):
        off, vals = _kjt(B, bag, g)
        coll.set_input(off.to(cuda), vals.to(cuda))
        pooled = coll.forward().float().cpu()
        torch.cuda.synchronize()
        coll.check()
        o, v = off.tolist(), vals.tolist()
        ref = np.stack([sum(_ref_row(store, ds.seed, k, dim, scale) for k in v[o[b]:o[b + 1]]) for b in range(B)])
        np.testing.assert_allclose(pooled.numpy(), ref, rtol=2e-2, atol=2e-4)
        grad = torch.randn(B, dim).to(torch.bfloat16)
        coll.grad_input.copy_(grad.to(cuda))
        coll.backward()
        gf = grad.float().numpy()
        for b in range(B):
            for k in v[o[b]:o[b + 1]]:
                store[k] = store[k] - lr * gf[b]
    torch.cuda.synchronize()
    keys, slots = ds.live()
    assert keys.numel() == len(store)
    w = coll.shard_view(0)[slots.long()].cpu().numpy()
    ref = np.stack([store[int(k)] for k in keys.cpu().tolist()])
    np.testing.assert_allclose(w, ref, rtol=1e-4, atol=1e-5)


def test_dynamic_eviction_and_rebuild_keep_lookups(cuda):
    dim = 32
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    C = 600
    spec = SparseTableSpec("d", C, dim, optimizer=opt, dynamic=True, hash_buckets=2048)
    B = 256
    coll = ShardedEmbeddingBagCollection([spec], B, max_bag_size=1, device=cuda, optimizer=opt, seed=2)
    ds = coll.dynamic.shards[0]
    g = torch.Generator().manual_seed(3)
    for _ in range(12):
        keys = torch.randint(0, KEY_SPACE, (B,), generator=g, dtype=torch.int64).to(torch.int32)
        off = torch.arange(B + 1, dtype=torch.int32)
        coll.set_input(off.to(cuda), keys.to(cuda))
        out = coll.forward().float()
        torch.cuda.synchronize()
        coll.check()
        # every bag holds one key: its pooled row is that key's slot row
        k_live, s_live = ds.live()
        slot_of = dict(zip(k_live.cpu().tolist(), s_live.cpu().tolist()))
        rows = torch.tensor([slot_of[int(k)] for k in keys.tolist()], device=cuda)
        torch.testing.assert_close(out, coll.shard_view(0)[rows].to(torch.bfloat16).float())
        coll.grad_input.copy_(torch.randn(B, dim, device=cuda).to(torch.bfloat16))
        coll.backward()
    # 12 x 256 distinct keys through 600 slots: thousands of evictions, tombstones reused by inserts
    tombs = int(ds.num_tomb.item())
    assert tombs == int((ds.keys == -2).sum())
    assert len(set(ds.live()[1].cpu().tolist())) == ds.live()[1].numel() <= C
    before = dict(zip(*[t.cpu().tolist() for t in ds.live()]))
    assert coll.dynamic.maintain(max_tomb_frac=0.0) == (1 if tombs > 0 else 0)
    after = dict(zip(*[t.cpu().tolist() for t in ds.live()]))
    assert before == after and int(ds.num_tomb.item()) == 0
    # lookups after the rebuild still find the resident keys
    live_keys = torch.tensor(list(after.keys())[:B], dtype=torch.int32)
    off = torch.arange(live_keys.numel() + 1, dtype=torch.int32)
    pad = B - live_keys.numel()
    if pad > 0:
        live_keys = torch.cat([live_keys, live_keys[:pad]])
        off = torch.arange(B + 1, dtype=torch.int32)
    coll.set_input(off.to(cuda), live_keys.to(cuda))
    out = coll.forward().float()
    torch.cuda.synchronize()
    coll.check()
    rows = torch.tensor([after[int(k)] for k in live_keys.tolist()], device=cuda)
    torch.testing.assert_close(out, coll.shard_view(0)[rows].to(torch.bfloat16).float())
