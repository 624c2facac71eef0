"""Host-DRAM tier: a table kept in pinned host memory with an HBM cache trains like the same
table fully resident in HBM (pooled outputs every step, weights and state at the end), up to
the last bit of the fp32 atomics of heavy rows, whose order varies from run to run."""
import numpy as np
import pytest
import torch

from flare_b200.data.synthetic import zipf_ids
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec

pytestmark = pytest.mark.gpu


def _kjt(B, vocabs, max_bag, g, dev):
    lens, vals = [], []
    for v in vocabs:
        ln = torch.randint(0, max_bag + 1, (B,), generator=g)
        lens.append(ln)
        vals.append(zipf_ids(int(ln.sum()), v, 1.05, g))
    lens = torch.cat(lens)
    off = torch.zeros(len(lens) + 1, dtype=torch.int32)
    torch.cumsum(lens, 0, out=off[1:])
    return off, torch.cat(vals)


@pytest.mark.parametrize("kind", ["rowwise_adagrad", "adam"])
def test_host_tier_matches_resident(cuda, kind):
    opt = SparseOptimizerConfig(kind=kind, learning_rate=0.05)
    vocabs = [1000, 20000]
    mk = lambda cache: [SparseTableSpec("a", vocabs[0], 64, optimizer=opt),  # noqa: E731
                        SparseTableSpec("b", vocabs[1], 64, optimizer=opt, cache_rows=cache)]
    B, bag = 256, 8
    ht_coll = ShardedEmbeddingBagCollection(mk(2500), B, max_bag_size=bag, device=cuda, optimizer=opt, seed=3)
    ref = ShardedEmbeddingBagCollection(mk(None), B, max_bag_size=bag, device=cuda, optimizer=opt, seed=3)
    tier = ht_coll.host_tier
    g = torch.Generator().manual_seed(0)
    for step in range(1, 13):
        off, vals = _kjt(B, vocabs, bag, g, "cpu")
        for c in (ht_coll, ref):
            c.set_input(off.to(cuda), vals.to(cuda))
        a, b = ht_coll.forward().clone(), ref.forward().clone()
        torch.cuda.synchronize()
        ht_coll.check()
        # equal up to the last bit of the heavy-row fp32 atomics (their order varies between runs)
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-5, msg=f"pooled differ at {step}")
        grad = torch.randn(B, ref.total_dim, device=cuda).to(torch.bfloat16)
        ht_coll.grad_input.copy_(grad)
        ref.grad_input.copy_(grad)
        ht_coll.backward()
        ref.backward()
    tier.flush()
    hs = tier.shards[0]
    assert hs.resident_rows() == hs.C  # the cache filled up, so rows were evicted and re-fetched
    j = [i for i, s in enumerate(ref.shards) if s.spec.name == "b"][0]
    f = ref.shard_fields(j)
    tol = dict(rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(hs.w, f["weight"].cpu(), **tol)
    if hs.h_row is not None:
        torch.testing.assert_close(hs.h_row, f["state_row"].cpu(), **tol)
    if hs.h_m is not None:
        torch.testing.assert_close(hs.h_m, f["state_m"].cpu(), **tol)
        torch.testing.assert_close(hs.h_v, f["state_v"].cpu(), **tol)
