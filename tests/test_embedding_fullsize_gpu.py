"""Full-size embedding backward (one B200): two 40M-row x 128 fp32 tables (5.1G elements each, so
every weight offset needs 64 bits), the benchmark's batch (8192 samples, bags U[1,64], Zipf(1.05) ids:
a Zipf head of thousands of occurrences per row).  The default hash-dedup backward and the
deterministic sorted backward update identical copies of the tables from the same pooled gradients;
the touched rows must agree (fp32 sums in another order), the untouched rows must be unchanged, and
the unique-row / heavy-row counts of both paths must match."""
import pytest
import torch

from flare_b200.data.synthetic import make_jagged
from flare_b200.sparse.collection import ShardedEmbeddingBagCollection
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec

pytestmark = pytest.mark.gpu

ROWS = 40_000_000


def test_hash_and_sorted_backward_agree_on_two_40M_row_tables(cuda):
    if torch.cuda.get_device_properties(cuda).total_memory < 100e9:
        pytest.skip("needs a GPU with at least 100 GB (two copies of two 20 GB tables)")
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    tables = [SparseTableSpec(f"t{i}", ROWS, 128, optimizer=opt) for i in range(2)]
    B, max_bag = 8192, 64
    g = torch.Generator().manual_seed(0)
    lengths = torch.randint(1, max_bag + 1, (2, B), generator=g)
    offs, vals = make_jagged(lengths, [ROWS, ROWS], 1.05, g)
    grad = (torch.randn(B, 256, generator=g) * 0.01).to(torch.bfloat16).to(cuda)
    results = []
    for det in (False, True):
        c = ShardedEmbeddingBagCollection(tables, B, max_bag_size=max_bag, device=cuda, seed=5, deterministic=det)
        assert c.hash_bwd == (not det)
        c.set_input(offs.to(cuda), vals.to(cuda), non_blocking=False)
        c.forward()
        c.grad_input.copy_(grad)
        c.backward()
        torch.cuda.synchronize()
        c.check()
        stats = c.last_step_stats()
        touched = torch.unique(vals.to(cuda).long() + torch.repeat_interleave(
            torch.tensor([0, ROWS], device=cuda), lengths.sum(1).to(cuda)))
        results.append((c, stats, touched))
    (a, sa, touched), (b, sb, _) = results
    assert sa["unique_rows"] == sb["unique_rows"] == touched.numel()
    assert sa["heavy_rows"] > 1000  # the Zipf head goes through the chunked path
    wa = a.weights.view(-1, 128)
    wb = b.weights.view(-1, 128)
    torch.testing.assert_close(wa[touched], wb[touched], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(a.state_row[touched], b.state_row[touched], rtol=1e-4, atol=1e-9)
    # rows nobody touched: identical initial values in both copies, and unchanged by either path
    probe = torch.randint(0, 2 * ROWS, (100_000,), device=cuda)
    untouched = probe[~torch.isin(probe, touched)]
    assert torch.equal(wa[untouched], wb[untouched])
    assert int(a.dirty_rows(0, 2 * ROWS).numel()) == touched.numel()
